#!/usr/bin/env python3
"""Converts the one model in the reference tree that the reference's own exporter wrote,
``tests/test-data/modules/fclayer/fclayer_architecture.json`` (an FCLayer module graph serialised
by FastOnnxModelBuilder as JSON), into ModelProto bytes: ``fclayer_architecture.onnx`` here.

    python tests/golden/gen_fclayer.py --reference PATH/TO/Shorokoo

The node list, names, op types, domains, attributes, opset imports (including the "Functions"
domain), graph input / output value infos and the model-local function ``fn_1`` are taken from the
fixture as they are. The fixture's JSON drops every tensor payload (``RawData`` / ``*Datas`` are
null), so the values of its Constant tensors are reconstructed from the graph itself and written
into ``fclayer_reconstructed.json`` beside the model:

* the shapes fed to the parameter initialiser ``fn_1`` (N3, N5) are the ``shrk_shape`` attributes
  of the calls that consume them ([5, 5] and [5]);
* N13 / N14 are the parameters' local model ids, the ``shrk_local_model_id`` attributes of the two
  calls ([1, 1] and [1, 2], as in ``fclayer_param_ids.txt``);
* N2 = [3, 1] turns an id into its position in the parameter sequence N8 (four empty placeholders,
  then the weight and the bias: positions 4 and 5);
* the Pad chains around the ids pad nothing: ReduceProd of equal one-element shapes (N15 = N18 =
  N31 = N34 = [2]) differ by 0, the leading pads N22 = N38 = [0], the pad values N9 = N11 = 0, the
  Unsqueeze axes N10 = N12 = [0];
* N7 is an empty float tensor (the placeholders);
* the fill value of ``fn_1``'s ConstantOfShape (the "InitSimple" initialiser) is taken as 0.5, so
  the module computes y = x W^T + b with W = 0.5 (5 x 5) and b = 0.5 (5).
"""
from __future__ import annotations

import argparse
import base64
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from shorokoo_b200.emit import onnx_writer as W  # noqa: E402

FIXTURE = "tests/test-data/modules/fclayer/fclayer_architecture.json"

CONSTANTS = {
    "N2": np.array([3, 1], np.int64),
    "N3": np.array([5, 5], np.int64),
    "N5": np.array([5], np.int64),
    "N7": np.zeros((0,), np.float32),
    "N9": np.array(0, np.int64),
    "N10": np.array([0], np.int64),
    "N11": np.array(0, np.int64),
    "N12": np.array([0], np.int64),
    "N13": np.array([1, 1], np.int64),
    "N14": np.array([1, 2], np.int64),
    "N15": np.array([2], np.int64),
    "N18": np.array([2], np.int64),
    "N22": np.array([0], np.int64),
    "N31": np.array([2], np.int64),
    "N34": np.array([2], np.int64),
    "N38": np.array([0], np.int64),
}
INIT_FILL = np.array([0.5], np.float32)   # fn_1's ConstantOfShape value


def _attr(a, node_name):
    t = a["Type"]
    if t == 1:
        return W.Attr(a["Name"], float(a["F"]), W.A_FLOAT)
    if t == 2:
        return W.Attr(a["Name"], int(a["I"]), W.A_INT)
    if t == 3:
        return W.Attr(a["Name"], base64.b64decode(a["S"] or ""), W.A_STRING)
    if t == 7:
        return W.Attr(a["Name"], [int(v) for v in (a["Ints"] or [])], W.A_INTS)
    if t == 6:
        return W.Attr(a["Name"], [float(v) for v in (a["Floats"] or [])], W.A_FLOATS)
    if t == 4:
        if node_name in CONSTANTS:
            arr = CONSTANTS[node_name]
        elif node_name == "N52":   # fn_1's ConstantOfShape
            arr = INIT_FILL
        else:
            raise ValueError(f"no reconstructed value for tensor attribute of {node_name}")
        dims = a["T"]["Dims"]
        if dims is not None:
            assert list(arr.shape) == list(dims), (node_name, arr.shape, dims)
        return W.Attr(a["Name"], W.Tensor("", arr, encoding="raw"), W.A_TENSOR)
    raise ValueError(f"attribute type {t} of {node_name}")


def _node(n):
    return W.Node(n["OpType"], list(n["Inputs"]), list(n["Outputs"]), name=n["Name"],
                  attrs=[_attr(a, n["Name"]) for a in n["Attributes"]], domain=n["Domain"] or "")


def _value_info(v):
    tt = (v["Type"] or {}).get("TensorType")
    meta = {m["Key"]: m["Value"] for m in v.get("MetadataProps") or []}
    if not tt:
        return W.ValueInfo(v["Name"], metadata=meta)
    shp = tt.get("Shape")
    dims = None
    if shp is not None:
        dims = [d["DimParam"] if d.get("DimParam") else int(d.get("DimValue", 0)) for d in shp["Dims"]]
    return W.ValueInfo(v["Name"], int(tt["ElemType"]), dims=dims, metadata=meta)


def convert(path: str) -> bytes:
    d = json.load(open(path))
    g = d["Graph"]
    graph = W.Graph(g.get("Name") or "FCLayer", [_node(n) for n in g["Nodes"]], [],
                    [_value_info(v) for v in g["Inputs"]], [_value_info(v) for v in g["Outputs"]])
    fns = []
    for f in d["Functions"]:
        fns.append(W.Function(f["Name"], f["Domain"], list(f["Inputs"]), list(f["Outputs"]),
                              [_node(n) for n in f["Nodes"]],
                              opsets={o["Domain"]: int(o["Version"]) for o in f["OpsetImports"]}))
    model = W.Model(graph, opsets={o["Domain"]: int(o["Version"]) for o in d["OpsetImports"]}, functions=fns,
                    ir_version=int(d["IrVersion"]), producer=d["ProducerName"])
    return model.encode()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    a = ap.parse_args()
    b = convert(os.path.join(a.reference, FIXTURE))
    with open(os.path.join(HERE, "fclayer_architecture.onnx"), "wb") as f:
        f.write(b)
    rec = {k: v.tolist() for k, v in CONSTANTS.items()}
    rec["fn_1.N52.value"] = INIT_FILL.tolist()
    with open(os.path.join(HERE, "fclayer_reconstructed.json"), "w") as f:
        json.dump(rec, f, indent=1)
    print(f"fclayer_architecture.onnx: {len(b)} bytes")


if __name__ == "__main__":
    main()
