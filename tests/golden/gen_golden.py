#!/usr/bin/env python3
"""Regenerates the golden fixtures in this directory from the reference's own Python references.

Run where the reference tree is checked out, giving its root:

    python tests/golden/gen_golden.py --reference PATH/TO/Shorokoo

* ``linear_pytorchref.npz`` — the reference's PyTorch Linear script
  (tests/pytorch-reference/linear.py, the generator behind NNLinearMatchesPyTorch,
  tests/Shorokoo.Tests/Modules/NNLibraryTestModules.cs:39-51) run as a subprocess on seeded weights.
* ``resnet18_torchref.npz`` — the reference's PyTorch twin of its ResNet-18 sample
  (tests/test-data/models/resnet18/make-reference-logits.py:29-78, used by
  RealCheckpointPredictionTests) loaded with the same seeded weights the emitter puts in the ONNX.

The fixtures hold the model inputs and the reference outputs; the weights are regenerated from the
seeds by ``shorokoo_b200.emit`` (the fixture keeps checksums of them so a drift in the generator is
caught).  The reference tree is read only here, never at test time.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from shorokoo_b200.emit import graphs  # noqa: E402

LINEAR_KW = dict(batch=3, widths=(16, 8), seed=5, bias_scale=0.5)
RESNET18_KW = dict(depth=18, batch=2, hw=(64, 64), seed=7, affine_scale=0.1)


def param_checksum(params) -> np.ndarray:
    keys = sorted(params)
    return np.array([float(np.float64(params[k]).sum()) for k in keys], np.float64)


def gen_linear(ref_root: str) -> None:
    from safetensors.numpy import save_file
    case = graphs.mlp(**LINEAR_KW)
    x = case.inputs[0][1]
    w = case.params["layers.0.weight"]
    b = case.params["layers.0.bias"]
    script = os.path.join(ref_root, "tests", "pytorch-reference", "linear.py")
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "linear.safetensors")
        save_file({"weight": w, "bias": b, "input": x}, path)
        out = subprocess.run([sys.executable, script, path], check=True, capture_output=True, text=True).stdout
    vals = [float(v) for v in re.findall(r"(-?\d+\.\d+)f", out)]
    y = np.array(vals, np.float32).reshape(x.shape[0], w.shape[0])
    np.savez(os.path.join(HERE, "linear_pytorchref.npz"), x=x, w=w, b=b, y=y,
             kwargs=repr(LINEAR_KW))
    print("linear:", y.shape, "max|y|", np.abs(y).max())


def gen_resnet18(ref_root: str) -> None:
    import torch
    spec = importlib.util.spec_from_file_location(
        "make_reference_logits",
        os.path.join(ref_root, "tests", "test-data", "models", "resnet18", "make-reference-logits.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    case = graphs.resnet(**RESNET18_KW)
    model = mod.ResNet18()
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in case.params.items()}
    for k in list(model.state_dict()):
        if k.endswith("num_batches_tracked"):
            sd[k] = torch.tensor(0)
    model.load_state_dict(sd, strict=True)
    model.eval()
    x = case.inputs[-1][1]
    with torch.no_grad():
        logits = model(torch.from_numpy(x)).numpy()
    np.savez(os.path.join(HERE, "resnet18_torchref.npz"), x=x, logits=logits,
             param_checksum=param_checksum(case.params), kwargs=repr(RESNET18_KW))
    print("resnet18:", logits.shape, "max|logit|", np.abs(logits).max())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    a = ap.parse_args()
    gen_linear(a.reference)
    gen_resnet18(a.reference)


if __name__ == "__main__":
    main()
