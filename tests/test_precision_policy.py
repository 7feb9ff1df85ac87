"""Host-side tests of the per-contraction precision policy (shorokoo_b200/csrc/precision.cpp): which
operand precision each fused Conv / Gemm gets in a bf16, TF32 and TF32x3 session. The policy keeps
the session's operand type on short or pooled chains (MLP-6, StackedLinear, ResNet) and, on a dense
chain of more than 16 contractions (RetinaNet's per-anchor outputs), moves the contractions past the
first 4 (bf16 session) to TF32 and those past the first 16 (TF32 session) to TF32x3. The accuracy
those choices buy is checked on the GPU (tests/test_gpu_models.py, test_gpu_tf32.py,
test_gpu_full_size.py)."""
from collections import Counter

import pytest

from shorokoo_b200.emit import graphs
from test_native_host import lower


def precisions(case):
    return [l.split("prec=")[1].split("/") for l in lower(case) if "prec=" in l]


@pytest.mark.parametrize("name,kw", [
    ("resnet50", dict(batch=2, hw=(64, 64))),
    ("resnet18", dict(batch=2, hw=(64, 64))),
    ("mlp", dict(batch=8)),
    ("stacked_linear", dict(batch=8)),
])
def test_short_or_pooled_chains_keep_the_session_precision(name, kw):
    p = precisions(graphs.build(name, **kw))
    assert p and all(x == ["bf16", "tf32", "tf32x3"] for x in p), Counter(map(tuple, p))


def test_retinanet_dense_chains_get_more_precise_operands():
    p = precisions(graphs.retinanet(batch=1, hw=(128, 160)))
    # lowered order: stem, then the first bottleneck's three convs (projection shortcut merged)
    assert p[:4] == [["bf16", "tf32", "tf32x3"]] * 4
    bf16_session = Counter(x[0] for x in p)
    tf32_session = Counter(x[1] for x in p)
    assert bf16_session == {"bf16": 4, "tf32": len(p) - 4}
    assert tf32_session == {"tf32": 16, "tf32x3": len(p) - 16}
    assert all(x[2] == "tf32x3" for x in p)


def test_shallow_detector_chain_still_counts_the_heads():
    # one bottleneck per stage: 1 + 12 backbone + FPN lateral and smooth + 5 head convs > 16
    p = precisions(graphs.retinanet(batch=1, hw=(128, 160), backbone_blocks=(1, 1, 1, 1)))
    assert Counter(x[0] for x in p)["bf16"] == 4
