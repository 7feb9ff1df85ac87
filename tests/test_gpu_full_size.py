"""GPU parity of the five benchmark configurations at their stated sizes, through the plugin
interface (Run with host buffers, so the micro-batch pipeline and its chunk plans run exactly as a
caller gets them), against the fp32 oracle at the bf16 accuracy gate (normwise max|gpu - ref| /
max|ref| per output, bf16 1e-2):

* StackedLinear n=1024 depth 8, batch 4096, seed 42      every row checked
* MLP 1024 -> 4096 x5 -> 1000, batch 8192, seed 1          every row checked
* ResNet-18 224x224, batch 256, seed 7                     every image checked
* ResNet-50 224x224, batch 512, seed 11 (the benchmark)    every image checked
* RetinaNet R50-FPN 800x1024, batch 16, seed 13            images at the pipeline's chunk seams,
                                                           the first and the last (the CPU oracle
                                                           takes seconds per image here)

The oracle runs on slices of the batch (every graph is per-sample in inference mode), so its
memory stays bounded. Besides the gate, the per-row error is checked on every compared row, so a
chunk of the pipelined run that went wrong cannot hide behind the max over the batch."""
import numpy as np
import pytest

from helpers import BF16_TOL, normwise_err, run_backend, run_oracle
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


def _oracle_rows(case, rows, chunk):
    """The oracle's outputs for the given batch rows, evaluated `chunk` rows at a time."""
    name, x = case.inputs[0]
    outs = None
    for i in range(0, len(rows), chunk):
        sub = graphs.ModelCase(case.name, case.model, [(name, x[rows[i:i + chunk]])], case.output_names, 0)
        r = run_oracle(sub)
        outs = r if outs is None else [np.concatenate([a, b]) for a, b in zip(outs, r)]
    return outs


def _check(case, rows, chunk, tol=BF16_TOL):
    got = run_backend(case)
    for g in got:
        assert np.all(np.isfinite(g)), f"{case.name}: non-finite output"
    ref = _oracle_rows(case, rows, chunk)
    errs = []
    for g, r, o in zip(got, ref, case.output_names):
        g = g[rows]
        e = normwise_err(g, r)
        errs.append(e)
        assert e <= tol, f"{case.name} output {o}: normwise error {e:.3e} > {tol:.1e}"
        # per row, against the batch-wide scale of the reference
        scale = float(np.abs(r).max())
        per_row = np.abs(g.astype(np.float64) - r).reshape(len(rows), -1).max(1) / scale
        assert per_row.max() <= tol, f"{case.name} output {o}: row {rows[int(per_row.argmax())]} at {per_row.max():.3e}"
    print(f"{case.name}: normwise error per output " + ", ".join(f"{e:.2e}" for e in errs) + f" (gate {tol:.0e})")
    return errs


def test_full_size_stacked_linear():
    case = graphs.build("stacked_linear")
    _check(case, np.arange(4096), 4096)


def test_full_size_mlp():
    case = graphs.build("mlp")
    _check(case, np.arange(8192), 2048)


def test_full_size_resnet18():
    case = graphs.build("resnet18")
    _check(case, np.arange(256), 64)


def test_full_size_resnet50():
    case = graphs.build("resnet50")
    _check(case, np.arange(512), 64)


def test_full_size_retinanet():
    case = graphs.build("retinanet")
    # Run's pipeline cuts the 16 images into chunks of 2 + 2 + 4 + 4 + 4
    _check(case, np.array([0, 1, 2, 4, 8, 15]), 1)
