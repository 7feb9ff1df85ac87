"""Parity report of the five benchmark graphs (small sizes): for each output, in both precisions,
the normwise error max|gpu - ref| / max|ref| against the fp32 oracle with its gate (bf16 1e-2,
TF32 and TF32x3 2e-3), and the elementwise pass rate |gpu - ref| <= tol * max(1e-3 * max|ref|, |ref|).

    python tests/parity_report.py            (needs a GPU; prints one line per output)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

from helpers import normwise_err, run_backend, run_oracle  # noqa: E402
from shorokoo_b200 import B200InferenceSessionFactory  # noqa: E402
from shorokoo_b200.emit import graphs  # noqa: E402

CASES = [
    ("stacked_linear", dict(batch=64)),
    ("mlp", dict(batch=96, widths=(256, 512, 512, 100))),
    ("resnet18", dict(batch=3, hw=(96, 96))),
    ("resnet50", dict(batch=2, hw=(64, 64), affine_scale=0.1)),
    ("retinanet", dict(batch=1, hw=(128, 160))),
]
GATES = {"bf16": 1e-2, "tf32": 2e-3, "tf32x3": 2e-3}


def elementwise_pass_rate(got, ref, tol):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    floor = 1e-3 * float(np.abs(ref).max()) if ref.size else 0.0
    ok = np.abs(got - ref) <= tol * np.maximum(floor, np.abs(ref))
    return float(ok.mean()) if ok.size else 1.0


def main():
    for name, kw in CASES:
        case = graphs.build(name, **kw)
        ref = run_oracle(case)
        for prec, gate in GATES.items():
            got = run_backend(case, factory=B200InferenceSessionFactory(num_devices=1, precision=prec))
            for g, r, o in zip(got, ref, case.output_names):
                e = normwise_err(g, r)
                rate = elementwise_pass_rate(g, r, gate)
                print(f"{name:15s} {prec} out {o:12s} normwise {e:.2e} (gate {gate:.0e}: "
                      f"{'pass' if e <= gate else 'FAIL'})  elementwise pass {100 * rate:.2f}%", flush=True)


if __name__ == "__main__":
    main()
