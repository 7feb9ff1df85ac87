"""GPU parity of the tcgen05 implicit-GEMM kernel and the memory-bound kernels against the oracle.

Shapes cover the edge cases of the tiling: M/N/K tails (not multiples of 128 / 64 / 64), tiny
problems (fewer tiles than SMs), every N-tile width, TMA-fed 1x1 convs, im2col-gathered spatial
convs (stride 2, SAME_UPPER asymmetric pads, dilation), the 4-channel stem path, the fused
epilogues (folded affine, residual, nearest-2x upsampled residual, ReLU, Sigmoid), and projection
shortcuts merged into the conv that adds them."""
import numpy as np
import pytest

from helpers import BF16_TOL, assert_close, conv_case, run_backend, run_oracle
from shorokoo_b200 import B200InferenceSessionFactory
from shorokoo_b200.emit import graphs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,n,relu", [
    (8, 16, 8, False), (300, 200, 100, True), (128, 64, 64, False), (1000, 96, 1000, True),
    (513, 1024, 4096, True), (64, 4096, 36, False), (2, 2048, 1000, False),
])
def test_gemm(m, k, n, relu):
    widths = (k, n) if not relu else (k, n, n)
    case = graphs.mlp(batch=m, widths=widths, seed=3, bias_scale=0.5)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert_close(got, ref, what=f"gemm {m}x{k}x{n}")


@pytest.mark.parametrize("kw", [
    dict(c=64, cout=64, k=1, pads=[0, 0, 0, 0]),                       # TMA-fed 1x1
    dict(c=64, cout=256, k=1, pads=[0, 0, 0, 0], bn=True, residual=True, relu=True),
    dict(c=64, cout=64, k=3, bn=True, relu=True),                       # gather 3x3, Cp % 64 == 0
    dict(c=24, cout=40, k=3, h=11, w=7),                                # Cp = 24: taps straddle K tiles
    dict(c=64, cout=128, k=3, stride=2, h=14, w=14),                    # stride 2
    dict(c=64, cout=128, k=1, stride=2, pads=[0, 0, 0, 0], h=14, w=14),  # strided 1x1 shortcut
    dict(c=3, cout=64, k=7, stride=2, pads=[3, 3, 3, 3], h=32, w=32, bn=True, relu=True),  # stem
    dict(c=32, cout=48, k=3, stride=2, auto_pad="SAME_UPPER", h=25, w=32),  # asymmetric pads
    dict(c=16, cout=16, k=3, dil=2, pads=[2, 2, 2, 2], h=12, w=12),
    dict(c=64, cout=720, k=3, auto_pad="SAME_UPPER", h=7, w=8, sigmoid=True),   # cls head
    dict(c=64, cout=36, k=3, auto_pad="SAME_UPPER", h=13, w=16),                # reg head
    dict(c=128, cout=64, k=1, pads=[0, 0, 0, 0], h=10, w=16, upsample_residual=True),  # FPN lateral
    dict(n=1, c=8, cout=8, k=3, h=1, w=1),
    # strided convs on <= 4 channels run over the 2x2 space-to-depth image
    dict(c=3, cout=64, k=7, stride=2, pads=[3, 2, 2, 3], h=31, w=33, bn=True, relu=True),
    dict(c=1, cout=16, k=3, stride=2, pads=[1, 1, 1, 1], h=9, w=12),
    dict(c=4, cout=24, k=5, stride=2, pads=[0, 0, 0, 0], h=17, w=16),
    dict(c=2, cout=8, k=3, stride=2, auto_pad="SAME_UPPER", h=10, w=7),
])
def test_conv(kw):
    case = conv_case(**kw)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert_close(got, ref, what=f"conv {kw}")


# Activations of at least 128 KiB whose channels come in 64s (or the 16-channel space-to-depth stem
# image) take the A operand by TMA in im2col mode; the step labels say which path ran.
@pytest.mark.parametrize("kw,path", [
    (dict(n=2, c=64, cout=64, k=3, h=32, w=32, bn=True, relu=True), "im2col"),
    (dict(n=3, c=128, cout=96, k=3, h=17, w=23), "im2col"),                       # M tail across images
    (dict(n=2, c=64, cout=128, k=3, stride=2, h=33, w=30), "im2col"),             # stride 2, odd H
    (dict(n=2, c=128, cout=256, k=1, stride=2, pads=[0, 0, 0, 0], h=28, w=28), "im2col"),
    (dict(n=2, c=64, cout=64, k=3, dil=2, pads=[2, 2, 2, 2], h=24, w=24), "im2col"),
    (dict(n=2, c=64, cout=48, k=3, stride=2, auto_pad="SAME_UPPER", h=25, w=32), "im2col"),
    (dict(n=2, c=64, cout=32, k=5, pads=[1, 2, 3, 0], h=20, w=30), "im2col"),     # asymmetric pads
    (dict(n=2, c=64, cout=64, k=3, h=32, w=32, bn=True, residual=True, relu=True), "im2col"),
    (dict(n=2, c=192, cout=256, k=3, h=16, w=16, sigmoid=True), "im2col"),        # 3 channel blocks
    (dict(n=2, c=3, cout=64, k=7, stride=2, pads=[3, 3, 3, 3], h=96, w=96, bn=True, relu=True), "im2col16"),
    (dict(n=2, c=3, cout=64, k=7, stride=2, pads=[3, 2, 2, 3], h=97, w=95), "im2col16"),
    (dict(n=2, c=1, cout=32, k=3, stride=2, pads=[1, 1, 1, 1], h=160, w=150), "im2col16"),   # 2x2 s2d taps
    (dict(n=2, c=4, cout=24, k=7, stride=2, pads=[2, 2, 2, 2], h=129, w=128), "im2col16"),
    (dict(n=2, c=4, cout=24, k=5, stride=2, pads=[0, 0, 0, 0], h=129, w=128), "s2d"),   # 3x3 taps: gather
])
def test_conv_im2col(kw, path):
    from shorokoo_b200 import B200InferenceSessionFactory
    case = conv_case(**kw)
    f = B200InferenceSessionFactory(num_devices=1)
    sess = f.CreateSession(case.model)
    feeds = {name: f.CreateTensor(arr) for name, arr in case.inputs}
    kinds = [k for k, _ in sess.profile(feeds, iters=1) if k.startswith("conv")]
    assert len(kinds) == 1 and path in kinds[0].split(), kinds
    outs = sess.Run(feeds, case.output_names)
    got = outs[0].numpy()
    for o in outs:
        o.Dispose()
    sess.Dispose()
    ref = run_oracle(case)[0]
    assert_close(got, ref, what=f"conv {kw}")


@pytest.mark.parametrize("n,c,h,w,k,stride,pads", [
    (2, 64, 112, 112, 3, 2, [1, 1, 1, 1]),    # the ResNet stem pool (3x3 fast path)
    (3, 32, 17, 23, 3, 2, [1, 0, 0, 1]),      # odd sizes, asymmetric pads
    (2, 16, 9, 9, 3, 1, [0, 0, 0, 0]),
    (2, 24, 10, 12, 2, 2, [0, 0, 0, 0]),      # general window
    (1, 5, 7, 7, 3, 2, [1, 1, 1, 1]),         # channels not a multiple of 8
])
def test_maxpool(n, c, h, w, k, stride, pads):
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase
    rng = np.random.Generator(np.random.PCG64(17))
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(18)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y = B.op("MaxPool", [xi], ceil_mode=0, dilations=[1, 1], kernel_shape=[k, k], pads=pads,
             strides=[stride, stride])
    ho = (h + pads[0] + pads[2] - k) // stride + 1
    wo = (w + pads[1] + pads[3] - k) // stride + 1
    B.shape[y] = (n, c, ho, wo)
    B.outputs.append(W.ValueInfo(y))
    case = ModelCase("maxpool", B.model("maxpool"), [(xi, x)], [y], 0)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert got.shape == (n, c, ho, wo)
    assert_close(got, ref, what=f"maxpool {n}x{c}x{h}x{w} k{k}/s{stride} {pads}")


def _stem_pool_case(n, h, w, seed=29, conv_output_too=False):
    """ResNet stem: conv 7x7/2 pad 3 over 3 channels + per-channel affine + ReLU + MaxPool 3x3/2 pad 1."""
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase, kaiming_normal
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n, 3, h, w), dtype=np.float32)
    B = Builder(seed + 1)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    wt = B.init(kaiming_normal(B.rng, (64, 3, 7, 7)), "w")
    y = B.conv(xi, wt, None, 7, 2, pads=[3, 3, 3, 3])
    sc = B.init((1 + 0.2 * B.rng.standard_normal((1, 64, 1, 1))).astype(np.float32), "s")
    sh = B.init((0.2 * B.rng.standard_normal((1, 64, 1, 1))).astype(np.float32), "t")
    y = B.unary("Relu", B.binary("Add", B.binary("Mul", y, sc), sh))
    p = B.op("MaxPool", [y], ceil_mode=0, dilations=[1, 1], kernel_shape=[3, 3], pads=[1, 1, 1, 1], strides=[2, 2])
    n_, c_, h_, w_ = B.shape[y]
    B.shape[p] = (n_, c_, (h_ - 1) // 2 + 1, (w_ - 1) // 2 + 1)
    # a 1x1 conv reads the pool, as ResNet's first bottleneck does (the pool output is then stored in
    # the bf16 operand layout the fused kernel writes)
    w2 = B.init(kaiming_normal(B.rng, (64, 64, 1, 1)), "w2")
    z = B.conv(p, w2, None, 1, 1, pads=[0, 0, 0, 0])
    B.outputs.append(W.ValueInfo(z))
    if conv_output_too:
        B.outputs.append(W.ValueInfo(y))
    outs = [z, y] if conv_output_too else [z]
    return ModelCase("stem_pool", B.model("stem_pool"), [(xi, x)], outs, 0)


# The stem conv and its 3x3/2 max pool run as one kernel when the conv output rows are even, at most
# 128 pixels wide and read only by the pool: each CTA computes a contiguous range of pool rows (with
# the halo conv row at the start of its range), so batches whose ranges start mid-image (3 x 32 pool
# rows over 148 CTAs: one each; 40 images: ranges across image boundaries) are covered. 230x230
# (odd conv rows) and 320x288 (144-pixel rows) take the separate conv and pool kernels.
@pytest.mark.parametrize("n,h,w,fused", [(2, 224, 224, True), (3, 64, 64, True), (5, 96, 128, True),
                                         (40, 64, 64, True), (1, 256, 96, True), (2, 230, 230, False),
                                         (1, 320, 288, False)])
def test_stem_with_fused_max_pool(n, h, w, fused):
    case = _stem_pool_case(n, h, w)
    f = B200InferenceSessionFactory(num_devices=1)
    sess = f.CreateSession(case.model)
    feeds = {nm: f.CreateTensor(a) for nm, a in case.inputs}
    kinds = [k for k, _ in sess.profile(feeds, iters=1)]
    assert any("+maxpool3x3/2" in k for k in kinds) == fused, kinds
    outs = sess.Run(feeds, case.output_names)
    got = outs[0].numpy()
    for o in outs:
        o.Dispose()
    sess.Dispose()
    ref = run_oracle(case)[0]
    assert got.shape == ref.shape
    assert_close(got, ref, what=f"stem + max pool {n}x3x{h}x{w}")
    if fused:   # against the separate conv and pool kernels (same weights, the conv output also read):
        # the two differ only in the conv's summation order, far below the gate
        other = run_backend(_stem_pool_case(n, h, w, conv_output_too=True))[0]
        assert_close(got, other, tol=2e-3, what="fused stem + pool vs separate kernels")


def test_stem_pool_not_fused_when_the_conv_output_is_also_read():
    case = _stem_pool_case(2, 64, 64, conv_output_too=True)
    got = run_backend(case)
    ref = run_oracle(case)
    for g, r in zip(got, ref):
        assert_close(g, r, what="stem with its conv output as a graph output")


# Split-K: contractions whose output tiles would fill under half the SMs run as slices of the
# reduction on separate CTAs (fp32 partials), then one reduce step adds the bias and residual and
# applies the activation and output type. Shapes: a batch-1 projection (1 M tile, 16 slices), a
# ragged M with ReLU, a 1x1 conv with a bf16 residual added in the reduce, a 3x3 conv with Sigmoid
# over 9 slices, a strided 3x3 512->512 conv over 12 slices, and TF32 operands.
@pytest.mark.parametrize("kind,kw,prec", [
    ("gemm", dict(batch=1, widths=(2048, 1000)), "bf16"),
    ("gemm", dict(batch=197, widths=(768, 3072, 768)), "bf16"),
    ("conv", dict(n=2, c=512, cout=128, k=1, pads=[0, 0, 0, 0], h=7, w=7, bn=True, residual=True, relu=True), "bf16"),
    ("conv", dict(n=1, c=128, cout=96, k=3, h=9, w=11, sigmoid=True), "bf16"),
    ("conv", dict(n=2, c=512, cout=512, k=3, stride=2, h=14, w=14, bn=True, relu=True), "bf16"),
    ("gemm", dict(batch=200, widths=(1024, 512)), "tf32"),
])
def test_split_k(kind, kw, prec):
    if kind == "gemm":
        case = graphs.mlp(seed=9, bias_scale=0.5, **kw)
    else:
        case = conv_case(seed=19, **kw)
    f = B200InferenceSessionFactory(num_devices=1, precision=prec)
    sess = f.CreateSession(case.model)
    feeds = {nm: f.CreateTensor(a) for nm, a in case.inputs}
    kinds = [k for k, _ in sess.profile(feeds, iters=1)]
    assert any(" split" in k for k in kinds) and any(k.startswith("split_reduce") for k in kinds), kinds
    outs = sess.Run(feeds, case.output_names)
    got = outs[0].numpy()
    for o in outs:
        o.Dispose()
    sess.Dispose()
    assert_close(got, run_oracle(case)[0], tol=BF16_TOL if prec == "bf16" else 2e-3, what=f"split-K {kind} {kw}")


def _halo_case(n, h, w, relu, seed=41):
    """Two chained 3x3 / stride 1 / pad 1 convs over 64 channels (+ per-channel affine, the first with
    ReLU when asked) and a 1x1 conv reading the second (so both 3x3 outputs are bf16 activations)."""
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase, kaiming_normal
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((n, 64, h, w), dtype=np.float32)
    B = Builder(seed + 1)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y = xi
    for i in range(2):
        wt = B.init(kaiming_normal(B.rng, (64, 64, 3, 3)), f"w{i}")
        y = B.conv(y, wt, None, 3, 1, pads=[1, 1, 1, 1])
        sc = B.init((1 + 0.2 * B.rng.standard_normal((1, 64, 1, 1))).astype(np.float32), f"s{i}")
        sh = B.init((0.2 * B.rng.standard_normal((1, 64, 1, 1))).astype(np.float32), f"t{i}")
        y = B.binary("Add", B.binary("Mul", y, sc), sh)
        if relu and i == 0:
            y = B.unary("Relu", y)
    w2 = B.init(kaiming_normal(B.rng, (32, 64, 1, 1)), "w2")
    z = B.conv(y, w2, None, 1, 1, pads=[0, 0, 0, 0])
    B.outputs.append(W.ValueInfo(z))
    return ModelCase("halo", B.model("halo"), [(xi, x)], [z], 0)


# 3x3 / stride 1 / pad 1 convs from 64 to 64 channels with bf16 outputs run from halo tiles (R rows x
# Wp pixels, one 4D TMA box of R + 2 input rows per tile, the taps read through row-shifted
# shared-memory descriptors): map widths giving tile widths 64 (R = 2), 32 (R = 4), 16 (R = 8) and
# 128 (R = 1), heights not a multiple of R, widths not a power of two, with and without ReLU; the
# 17x23 map (too many junk pixels in 32-wide tiles) takes the im2col kernel.
@pytest.mark.parametrize("n,h,w,relu,halo", [(2, 56, 56, True, True), (3, 28, 28, True, True),
                                             (2, 14, 14, False, True), (2, 30, 50, True, True),
                                             (4, 9, 100, True, True), (2, 17, 23, True, False)])
def test_conv3x3_halo_tiles(n, h, w, relu, halo):
    case = _halo_case(n, h, w, relu)
    f = B200InferenceSessionFactory(num_devices=1)
    sess = f.CreateSession(case.model)
    feeds = {nm: f.CreateTensor(a) for nm, a in case.inputs}
    kinds = [k for k, _ in sess.profile(feeds, iters=1)]
    assert sum(k.endswith(" halo") for k in kinds) == (2 if halo else 0), kinds
    outs = sess.Run(feeds, case.output_names)
    got = outs[0].numpy()
    for o in outs:
        o.Dispose()
    sess.Dispose()
    assert_close(got, run_oracle(case)[0], what=f"3x3 halo convs {n}x64x{h}x{w}")


def test_maxpool_and_gap():
    case = graphs.resnet(depth=18, batch=2, hw=(40, 40), seed=5, include_top=False)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert got.shape == (2, 512, 1, 1)
    assert_close(got, ref, what="resnet18 trunk + GAP")


def _conv(B, x, cin, cout, k, relu=False, res=None):
    from shorokoo_b200.emit.graphs import kaiming_normal
    w = B.init(kaiming_normal(B.rng, (cout, cin, k, k)), "w")
    b = B.init((0.3 * B.rng.standard_normal(cout)).astype(np.float32), "b")
    y = B.op("Conv", [x, w, b], auto_pad="NOTSET", dilations=[1, 1], group=1, kernel_shape=[k, k],
             pads=[k // 2] * 4, strides=[1, 1])
    if res is not None:
        y = B.op("Add", [y, res])
    return B.op("Relu", [y]) if relu else y


# Convs whose bf16 output feeds another conv and whose tile is 64 columns wide split each 32-row
# output slab between the TMEM quarter's two epilogue warps (one 32-column half each): ragged
# channel counts (48: the second half is partly outside; 24: the second half is empty). The middle
# conv's bf16 residual is added by the tensor core as one extra k-tile per 64 channels (96: the
# second residual k-tile is partly outside the tensor; 200: four of them, the last partly outside).
# The 8-image 64x64 case takes 256-column tiles with too few pipeline stages for full output slabs,
# so its bf16 output also goes out in 32-column halves (the last 64-column slab's first half partly
# outside the 200 channels, its second half empty).
@pytest.mark.parametrize("cmid,n,h,w", [(64, 2, 48, 40), (48, 2, 48, 40), (24, 2, 48, 40), (96, 2, 48, 40),
                                        (200, 2, 48, 40), (200, 8, 64, 64)])
def test_conv_chain_64_column_tiles(cmid, n, h, w):
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase
    rng = np.random.Generator(np.random.PCG64(23))
    c = 32
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(24)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y1 = _conv(B, xi, c, cmid, 3, relu=True)
    y2 = _conv(B, y1, cmid, cmid, 1, relu=True, res=y1)
    y3 = _conv(B, y2, cmid, 16, 3)
    for t, ch in ((y1, cmid), (y2, cmid), (y3, 16)):
        B.shape[t] = (n, ch, h, w)
    B.outputs.append(W.ValueInfo(y3))
    case = ModelCase("conv_chain", B.model("conv_chain"), [(xi, x)], [y3], 0)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert got.shape == (n, 16, h, w)
    assert_close(got, ref, what=f"conv chain through {cmid} channels")


# 256-column bf16 tiles that stream their weights run on CTA pairs (clusters of two, cta_group::2
# MMAs of 256 x 256): a 3x3 conv through TMA im2col to 320 channels (the second column tile holds 64
# of them), a 1x1 conv through row-matrix TMA, and a 1x1 conv whose residual the pair's tensor core
# adds (each CTA holding half of the identity operand), each feeding another conv; then 3x3 convs to
# 128 channels (one-SM 128-column tiles: pairs of 256 x 128 measured slower, their single MMA issuer
# the limit), the second with a residual.
def test_cta_pair_convs():
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase
    rng = np.random.Generator(np.random.PCG64(31))
    n, c, h, w = 8, 64, 64, 64
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(32)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    y1 = _conv(B, xi, c, 320, 3, relu=True)
    y2 = _conv(B, y1, 320, 256, 1, relu=True)
    y3 = _conv(B, y2, 256, 256, 1, relu=True, res=y2)
    y4 = _conv(B, y3, 256, 128, 3, relu=True)
    y5 = _conv(B, y4, 128, 128, 3, relu=True, res=y4)
    y6 = _conv(B, y5, 128, 16, 3)
    for t, ch in ((y1, 320), (y2, 256), (y3, 256), (y4, 128), (y5, 128), (y6, 16)):
        B.shape[t] = (n, ch, h, w)
    B.outputs.append(W.ValueInfo(y6))
    case = ModelCase("pair_chain", B.model("pair_chain"), [(xi, x)], [y6], 0)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert got.shape == (n, 16, h, w)
    assert_close(got, ref, what="conv chain on CTA pairs")


def _conv_s(B, x, cin, cout, k, stride=1, relu=False, res=None):
    from shorokoo_b200.emit.graphs import kaiming_normal
    w = B.init(kaiming_normal(B.rng, (cout, cin, k, k)), "w")
    b = B.init((0.3 * B.rng.standard_normal(cout)).astype(np.float32), "b")
    y = B.op("Conv", [x, w, b], auto_pad="NOTSET", dilations=[1, 1], group=1, kernel_shape=[k, k],
             pads=[k // 2] * 4, strides=[stride, stride])
    if res is not None:
        y = B.op("Add", [y, res])
    return B.op("Relu", [y]) if relu else y


# A bottleneck whose 1x1 projection shortcut (stride 1, or stride 2 over an odd-sized map) is merged
# into the last 1x1 conv: one GEMM over both operands' channels, the shortcut's input read through
# a second tensor map (row matrix, or im2col at the shortcut's stride).
# The 8-image cases with 256 middle channels (K = 256 + 128 streamed weights, 32768 output pixels)
# run the merged conv on CTA pairs.
@pytest.mark.parametrize("stride,h,w,cout,n,mid", [(1, 12, 10, 256, 2, 64), (2, 15, 13, 256, 2, 64),
                                                   (2, 16, 16, 192, 2, 64), (1, 64, 64, 256, 8, 256),
                                                   (2, 128, 128, 256, 8, 256)])
def test_merged_projection_shortcut(stride, h, w, cout, n, mid):
    from shorokoo_b200.emit import onnx_writer as W
    from shorokoo_b200.emit.graphs import Builder, ModelCase
    rng = np.random.Generator(np.random.PCG64(31))
    c = 128
    x = rng.standard_normal((n, c, h, w), dtype=np.float32)
    B = Builder(32)
    xi = B.graph_input(W.FLOAT, 4, x.shape)
    ho, wo = (h - 1) // stride + 1, (w - 1) // stride + 1
    a = _conv_s(B, xi, c, mid, 1, relu=True)
    bb = _conv_s(B, a, mid, mid, 3, stride=stride, relu=True)
    sc = _conv_s(B, xi, c, cout, 1, stride=stride)
    y = _conv_s(B, bb, mid, cout, 1, relu=True, res=sc)
    z = _conv_s(B, y, cout, 16, 1)   # y feeds a conv, so the merged conv writes bf16
    for t, ch, hh, ww in ((a, mid, h, w), (bb, mid, ho, wo), (sc, cout, ho, wo), (y, cout, ho, wo), (z, 16, ho, wo)):
        B.shape[t] = (n, ch, hh, ww)
    B.outputs.append(W.ValueInfo(z))
    case = ModelCase("merged_shortcut", B.model("merged_shortcut"), [(xi, x)], [z], 0)
    got = run_backend(case)[0]
    ref = run_oracle(case)[0]
    assert got.shape == (n, 16, ho, wo)
    assert_close(got, ref, what=f"bottleneck with merged stride-{stride} shortcut {h}x{w}")
