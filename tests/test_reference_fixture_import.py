"""Import of the one model the reference's own exporter wrote (tests/test-data/modules/fclayer/
fclayer_architecture.json, an FCLayer module graph), converted to ModelProto bytes by
tests/golden/gen_fclayer.py (its tensor payloads, dropped by the JSON dump, reconstructed there).

It carries what the stand-in emitter does not: the "Functions" opset import and a model-local
function ``fn_1`` (the parameter initialiser, a ConstantOfShape) called with the reference's
``shrk_*`` attributes, the module's parameters gathered in a SequenceConstruct and picked by
SequenceAt at indices computed from int64 Pad / Mul / ReduceSum / ReduceProd chains, Identity
wrappers, and a rank-1 graph input with a symbolic dim feeding MatMul(x, Transpose(W)) + b.

The module's input has 5 elements, so the backend treats it as a plan-time value (inputs of at most
16 elements key the plan cache, like the reference's [Hyper] scalars): the importer parses the model,
inlines the function and folds the whole graph, parameter machinery and all, on the host; the
result is a host output of the plan. The oracle interprets the same bytes; Run returns the same
result (y = x W^T + b with W = 0.5 and b = 0.5)."""
import os

import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, run_backend, run_oracle
from shorokoo_b200.emit.graphs import ModelCase
from test_native_host import lower

HERE = os.path.dirname(os.path.abspath(__file__))
MODEL = os.path.join(HERE, "golden", "fclayer_architecture.onnx")


def _case():
    with open(MODEL, "rb") as f:
        model = f.read()
    x = np.random.Generator(np.random.PCG64(3)).standard_normal(5, dtype=np.float32)
    return ModelCase("fclayer", model, [("N1_T0", x)], ["N50_T0"], 25)


def test_fixture_folds_on_the_host():
    lines = lower(_case())
    ops = [l.split()[0] for l in lines if not l.startswith(("output", "separable"))]
    assert ops == [], lines
    assert "output [5] host" in lines


def test_oracle_reads_the_fixture():
    case = _case()
    y = run_oracle(case)[0]
    x = case.inputs[0][1]
    np.testing.assert_allclose(y, np.full(5, 0.5 * x.sum() + 0.5, np.float32), rtol=1e-6)


@pytest.mark.gpu
def test_backend_runs_the_fixture():   # (a CUDA device is needed to open a session)
    case = _case()
    assert_close(run_backend(case)[0], run_oracle(case)[0], tol=BF16_TOL, what="fclayer fixture")
