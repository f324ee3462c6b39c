"""GEMM kernels (tcgen05 tensor-core path and the SIMT path) against a plain
fp32 PyTorch reference of the same product."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from dlvk_b200 import _ext

    return _ext.C()


def _ref(a, b, bias=None, act=0, alpha=1.0):
    c = alpha * (a.float() @ b.float())
    if bias is not None:
        c = c + bias.float()
    if act == 1:
        c = torch.relu(c)
    return c


def _check(out, ref, tol):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} (scale {scale})"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (300, 200, 100), (1024, 1024, 1024),
                                   (8192 // 4, 3072, 1024), (32, 128, 784), (129, 136, 72)])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_tc_layouts(M, N, K, a_t, b_t, out_dtype):
    C = _C()
    torch.manual_seed(0)
    dev = "cuda"
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(K, N, device=dev).bfloat16()
    A = a.t().contiguous().t() if a_t else a  # M-major view when a_t
    B = b.t().contiguous().t() if b_t else b  # K-major ([N,K] storage) when b_t
    if not C.gemm_tc_ok(A, B):
        pytest.skip("layout not eligible for the tensor-core path")
    out = C.gemm(A, B, force_path=1, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    # bf16 output: one rounding to 8 significant bits; fp32 output: only the
    # fp32 accumulation order differs from the reference product
    _check(out, _ref(a, b), 1e-2 if out_dtype == torch.bfloat16 else 1e-4)


def _padded(rows, cols, transposed, dtype):
    """A [rows, cols] operand whose row stride is padded to a multiple of 8
    elements (16-byte aligned rows for TMA), stored row-major, or stored
    transposed ([cols, rows(padded)]) and viewed back when `transposed`."""
    if transposed:
        st = torch.randn(cols, (rows + 7) // 8 * 8, device="cuda").to(dtype)
        return st[:, :rows].t()
    st = torch.randn(rows, (cols + 7) // 8 * 8, device="cuda").to(dtype)
    return st[:, :cols]


# Tile edges (128-row tiles, 128/256-column tiles, 64-deep k-blocks) +- 1.
@pytest.mark.parametrize("M,N,K", [(127, 128, 64), (128, 129, 63), (129, 255, 65), (255, 256, 127),
                                   (256, 257, 128), (257, 383, 129), (383, 384, 191), (385, 512, 257),
                                   (1, 16, 1), (2, 17, 3)])
@pytest.mark.parametrize("a_t", [False, True])
def test_gemm_tc_tile_edges(M, N, K, a_t):
    C = _C()
    torch.manual_seed(M + N + K)
    A = _padded(M, K, a_t, torch.bfloat16)
    B = _padded(K, N, False, torch.bfloat16)
    assert C.gemm_tc_ok(A, B)
    out = C.gemm(A, B, out_dtype=torch.float32, force_path=1)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(out, _ref(A, B), 1e-4)


def _ref64(a, b):
    return a.double() @ b.double()


@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (300, 200, 100), (129, 136, 72), (1024, 1024, 4096),
                                   (2048, 512, 1024)])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_gemm_fp32_tensor_cores(M, N, K, a_t, b_t):
    """fp32 operands on tcgen05 kind::tf32: 3xTF32 within 1e-5 of an fp64
    product (fp32-class accuracy), one TF32 pass within 5e-3."""
    C = _C()
    torch.manual_seed(M * 7 + N + K)
    A = _padded(M, K, a_t, torch.float32)
    B = _padded(K, N, b_t, torch.float32)
    assert C.gemm_tf32_ok(A, B)
    ref = _ref64(A, B)
    old = C.fp32_gemm_mode()
    try:
        for mode, tol in ((3, 1e-5), (1, 5e-3)):
            C.set_fp32_gemm_mode(mode)
            out = C.gemm(A, B, force_path=1)
            torch.cuda.synchronize()
            assert C.read_device_error(True) == 0
            rel = ((out.double() - ref).norm() / ref.norm()).item()
            assert rel < tol, (mode, rel)
        # the full epilogue on the last 3xTF32 pass: alpha, beta, bias, ReLU
        C.set_fp32_gemm_mode(3)
        bias = torch.randn(N, device="cuda")
        acc = torch.randn(M, N, device="cuda")
        want = torch.relu(0.5 * ref + 1.0 * acc.double() + bias.double())
        C.gemm(A, B, bias=bias, act=1, alpha=0.5, beta=1.0, out=acc, force_path=1)
        rel = ((acc.double() - want).norm() / want.norm()).item()
        assert rel < 1e-5, rel
    finally:
        C.set_fp32_gemm_mode(old)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_tc_epilogue(out_dtype):
    C = _C()
    torch.manual_seed(1)
    M, N, K = 512, 384, 256
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    bias = torch.randn(N, device="cuda")
    out = C.gemm(a, b, bias=bias, act=1, alpha=0.5, out_dtype=out_dtype, force_path=1)
    _check(out, _ref(a, b, bias, 1, 0.5), 2e-2)
    # beta accumulation into an f32 output (gradient accumulation)
    acc = torch.randn(M, N, device="cuda")
    ref = acc + a.float() @ b.float()
    C.gemm(a, b, beta=1.0, out=acc, force_path=1)
    _check(acc, ref, 2e-2)


def test_gemm_tc_batched():
    C = _C()
    torch.manual_seed(2)
    Bt, M, N, K = 6, 256, 192, 64
    a = torch.randn(Bt, M, K, device="cuda").bfloat16()
    b = torch.randn(Bt, K, N, device="cuda").bfloat16()
    out = C.gemm(a, b, force_path=1, out_dtype=torch.float32)
    _check(out, a.float() @ b.float(), 2e-2)
    # Q K^T style: B given as a transposed view of [Bt, N, K]
    kk = torch.randn(Bt, N, K, device="cuda").bfloat16()
    out2 = C.gemm(a, kk.transpose(1, 2), force_path=1, out_dtype=torch.float32)
    _check(out2, a.float() @ kk.float().transpose(1, 2), 2e-2)


def test_gemm_tc_persistent_small_grid():
    """Few CTAs loop over many tiles: exercises the TMEM double buffer and ring phases."""
    C = _C()
    a = torch.randn(2048, 512, device="cuda").bfloat16()
    b = torch.randn(512, 1024, device="cuda").bfloat16()
    out = C.gemm(a, b, force_path=1, max_ctas=3)
    _check(out, _ref(a, b), 2e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(32, 10, 128), (33, 47, 784), (257, 130, 65)])
def test_gemm_simt(dtype, M, N, K):
    C = _C()
    a = torch.randn(M, K, device="cuda").to(dtype)
    b = torch.randn(N, K, device="cuda").to(dtype).t()  # strided view
    bias = torch.randn(N, device="cuda")
    out = C.gemm(a, b, bias=bias, act=1, force_path=2, out_dtype=torch.float32)
    _check(out, _ref(a, b, bias, 1), 1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_tc_splitk_epilogues(out_dtype):
    """Few output tiles and a long K select split-K (fp32 workspace + reduce)."""
    C = _C()
    torch.manual_seed(3)
    M, N, K = 256, 384, 8192
    a = torch.randn(K, M, device="cuda").bfloat16().t()       # M-major (like X^T in dW)
    b = torch.randn(K, N, device="cuda").bfloat16()
    bias = torch.randn(N, device="cuda")
    res = torch.randn(M, N, device="cuda").to(out_dtype)
    mask = torch.randn(M, N, device="cuda").to(out_dtype)
    out = C.gemm(a, b, bias=bias, act=1, alpha=0.25, residual=res, relu_mask=mask, out_dtype=out_dtype, force_path=1)
    ref = torch.relu(0.25 * (a.float() @ b.float()) + bias + res.float())
    ref = torch.where(mask.float() > 0, ref, torch.zeros_like(ref))
    _check(out, ref, 2e-2)
    acc = torch.randn(M, N, device="cuda")
    ref2 = acc + a.float() @ b.float()
    C.gemm(a, b, beta=1.0, out=acc, force_path=1)
    _check(acc, ref2, 2e-2)


@pytest.mark.parametrize("epi", ["bias", "relu", "bias_relu", "residual", "mask"])
def test_gemm_tc_epilogue_variants(epi):
    C = _C()
    torch.manual_seed(4)
    M, N, K = 1000, 1040, 320
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    kw = {}
    ref = a.float() @ b.float()
    if "bias" in epi:
        kw["bias"] = torch.randn(N, device="cuda")
        ref = ref + kw["bias"]
    if epi == "residual":
        kw["residual"] = torch.randn(M, N, device="cuda").bfloat16()
        ref = ref + kw["residual"].float()
    if "relu" in epi:
        kw["act"] = 1
        ref = torch.relu(ref)
    if epi == "mask":
        kw["relu_mask"] = torch.randn(M, N, device="cuda").bfloat16()
        ref = torch.where(kw["relu_mask"].float() > 0, ref, torch.zeros_like(ref))
    out = C.gemm(a, b, force_path=1, **kw)
    _check(out, ref, 2e-2)


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 320), (1000, 520, 1024), (4096, 4096, 512)])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("epi", ["none", "bias_relu", "residual"])
def test_gemm_tc_pair_matches_single(M, N, K, a_t, b_t, epi):
    """The CTA-pair (cta_group::2) kernel against the single-CTA kernel and
    the fp32 reference."""
    C = _C()
    torch.manual_seed(3)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    A = a.t().contiguous().t() if a_t else a
    B = b.t().contiguous().t() if b_t else b
    kw = {}
    ref = a.float() @ b.float()
    if epi == "bias_relu":
        kw = dict(bias=torch.randn(N, device="cuda"), act=1)
        ref = torch.relu(ref + kw["bias"])
    elif epi == "residual":
        kw = dict(residual=torch.randn(M, N, device="cuda").bfloat16())
        ref = ref + kw["residual"].float()
    outs = []
    for on in (True, False):
        C.gemm_set_pair(on)
        try:
            outs.append(C.gemm(A, B, force_path=1, **kw))
        finally:
            C.gemm_set_pair(True)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(outs[0], ref, 2e-2)
    _check(outs[1], ref, 2e-2)
    assert (outs[0].float() - outs[1].float()).abs().max().item() <= 2e-2 * (ref.abs().max().item() + 1e-6)


def test_gemm_tc_pair_persistent_one_pair():
    C = _C()
    a = torch.randn(4096, 512, device="cuda").bfloat16()
    b = torch.randn(512, 2048, device="cuda").bfloat16()
    out = C.gemm(a, b, force_path=1, max_ctas=2)  # one CTA pair walks all 128 tiles
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(out, _ref(a, b), 2e-2)


@pytest.mark.parametrize("M,N", [(1024, 1024), (512, 3072), (2048, 512)])
def test_gemm_tc_pair_splitk_wgrad_shapes(M, N):
    """Weight-gradient shapes (few output tiles, K = 8192 tokens, both
    operands M/N-major) take split-K on the CTA-pair kernel; with beta = 1 the
    reduce accumulates into the existing gradient."""
    C = _C()
    torch.manual_seed(5)
    K = 8192
    a = torch.randn(K, M, device="cuda").bfloat16().t()  # X^T
    b = torch.randn(K, N, device="cuda").bfloat16()      # dY
    out = C.gemm(a, b, out_dtype=torch.float32, force_path=1)
    _check(out, a.float() @ b.float(), 2e-2)
    acc = torch.randn(M, N, device="cuda")
    ref = acc + a.float() @ b.float()
    C.gemm(a, b, beta=1.0, out=acc, force_path=1)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(acc, ref, 2e-2)


@pytest.mark.parametrize("M,N", [(1000, 1000), (384, 2056)])
def test_gemm_tc_splitk_reduce_into_strided_fp32(M, N):
    """Split-K partials added into an fp32 output that is a column window of a
    wider buffer (ragged M and N, alpha != 1): the columns outside the window
    and the rows' padding stay untouched, beta = 0 overwrites, beta = 1 adds."""
    C = _C()
    torch.manual_seed(6)
    K = 8192
    a = torch.randn(K, M, device="cuda").bfloat16().t()
    b = torch.randn(K, N, device="cuda").bfloat16()
    big = torch.full((M, N + 68), 7.0, device="cuda")
    out = big[:, 4:4 + N]
    ref = 0.5 * (a.float() @ b.float())
    C.gemm(a, b, alpha=0.5, out=out, force_path=1)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(out, ref, 2e-2)
    assert torch.all(big[:, :4] == 7.0) and torch.all(big[:, 4 + N:] == 7.0)
    C.gemm(a, b, alpha=0.5, beta=1.0, out=out, force_path=1)
    torch.cuda.synchronize()
    _check(out, 2 * ref, 2e-2)
    assert torch.all(big[:, :4] == 7.0) and torch.all(big[:, 4 + N:] == 7.0)


def _wide(C, mode):
    C.gemm_set_wide(mode)


@pytest.mark.parametrize("M,N,K", [(512, 1024, 256), (1000, 1000, 320), (768, 1536, 1024)])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("epi", ["none", "bias_relu", "residual", "mask"])
def test_gemm_tc_wide_pair_tile(M, N, K, a_t, b_t, epi):
    """The 256 x 512 CTA-pair tile (two N = 256 MMAs per k-step, one TMEM
    buffer), forced on, against the fp32 reference and the 256-wide tile."""
    C = _C()
    torch.manual_seed(7)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    A = a.t().contiguous().t() if a_t else a
    B = b.t().contiguous().t() if b_t else b
    kw = {}
    ref = a.float() @ b.float()
    if epi == "bias_relu":
        kw = dict(bias=torch.randn(N, device="cuda"), act=1)
        ref = torch.relu(ref + kw["bias"])
    elif epi == "residual":
        kw = dict(residual=torch.randn(M, N, device="cuda").bfloat16())
        ref = ref + kw["residual"].float()
    elif epi == "mask":
        kw = dict(relu_mask=torch.randn(M, N, device="cuda").bfloat16())
        ref = torch.where(kw["relu_mask"].float() > 0, ref, torch.zeros_like(ref))
    try:
        _wide(C, 2)
        assert C.gemm_plan(A, B)[0] == 512
        wide = C.gemm(A, B, force_path=1, **kw)
        _wide(C, 0)
        assert C.gemm_plan(A, B)[0] != 512
        narrow = C.gemm(A, B, force_path=1, **kw)
    finally:
        _wide(C, 1)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(wide, ref, 2e-2)
    _check(narrow, ref, 2e-2)


def test_gemm_tc_wide_pair_tile_splitk_batched_persistent():
    """Wide tile with split-K partials added into fp32 C, with 4-D batching,
    and with one CTA pair walking 16 tiles through its single TMEM buffer."""
    C = _C()
    torch.manual_seed(8)
    try:
        _wide(C, 2)
        a = torch.randn(8192, 1024, device="cuda").bfloat16().t()     # M-major, like X^T
        b = torch.randn(8192, 1024, device="cuda").bfloat16()
        plan = C.gemm_plan(a, b, True)
        assert plan[0] == 512 and plan[1] > 1
        out = C.gemm(a, b, out_dtype=torch.float32, force_path=1)
        _check(out, a.float() @ b.float(), 2e-2)
        acc = torch.randn(1024, 1024, device="cuda")
        ref = acc + a.float() @ b.float()
        C.gemm(a, b, beta=1.0, out=acc, force_path=1)
        _check(acc, ref, 2e-2)
        x = torch.randn(2, 3, 512, 128, device="cuda").bfloat16()
        w = torch.randn(2, 3, 128, 1024, device="cuda").bfloat16()
        _check(C.gemm(x, w, force_path=1, out_dtype=torch.float32), x.float() @ w.float(), 2e-2)
        a2 = torch.randn(1024, 384, device="cuda").bfloat16()
        b2 = torch.randn(384, 4096, device="cuda").bfloat16()
        assert C.gemm_plan(a2, b2, False, 2)[0] == 512
        _check(C.gemm(a2, b2, force_path=1, max_ctas=2), a2.float() @ b2.float(), 2e-2)
    finally:
        _wide(C, 1)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0


@pytest.mark.parametrize("M,N,K,out_dtype", [(512, 1024, 256, torch.bfloat16), (8192, 4096, 1024, torch.bfloat16),
                                             (256, 384, 320, torch.float32), (200, 1000, 128, torch.bfloat16)])
def test_gemm_tc_fused_colsum(M, N, K, out_dtype):
    """Column sums of a ReLU-masked dX = dY W^T (the previous layer's bias
    gradient), fused into the epilogue where M and N are multiples of 32 and a
    separate pass otherwise; overwrite and accumulate."""
    C = _C()
    torch.manual_seed(9)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(N, K, device="cuda").bfloat16().t()
    mask = torch.randn(M, N, device="cuda").to(out_dtype)
    ref = torch.where(mask.float() > 0, a.float() @ b.float(), torch.zeros(M, N, device="cuda"))
    cs = torch.full((N,), 5.0, device="cuda")
    out = C.gemm(a, b, relu_mask=mask, out_dtype=out_dtype, force_path=1, colsum_out=cs, colsum_scale=0.5)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
    _check(out, ref, 2e-2)
    _check(cs, 0.5 * ref.sum(0), 4e-3)
    C.gemm(a, b, relu_mask=mask, out_dtype=out_dtype, force_path=1, colsum_out=cs, colsum_accumulate=True)
    _check(cs, 1.5 * ref.sum(0), 4e-3)


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (1024, 1024, 512), (300, 200, 100), (96, 1000, 64)])
@pytest.mark.parametrize("force_path", [0, 2])  # 0: tensor cores where the layout allows, 2: SIMT
def test_gemm_relu_bitmask(M, N, K, force_path):
    """The forward GEMM writes one bit per output (> 0 after bias + ReLU); the
    backward GEMM zeroes its output where the bit is clear, with the fused
    column sums, and matches the same backward through a bf16 mask."""
    from dlvk_b200.ops.core import _unpack_bits, relu_bits_like

    C = _C()
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = (torch.randn(K, N, device="cuda", generator=g) * 0.1).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    bits = relu_bits_like(M, N, "cuda")
    f = C.gemm(a, b, bias=bias, act=1, force_path=force_path, relu_bits_out=bits)
    ref = _ref(a, b, bias, act=1)
    _check(f, ref, 1e-2)
    pos = _unpack_bits(bits, N)
    # bits agree with the reference wherever the output is not within rounding of zero
    sure = (ref.abs() > 1e-3 * ref.abs().max())
    assert torch.equal(pos[sure], (ref > 0)[sure])
    # padding bits past N are clear
    if N % 32:
        tail = (bits[:, -1].to(torch.int64) & 0xFFFFFFFF) >> (N % 32)
        assert int(tail.abs().sum()) == 0
    # backward: dF = (G W^T) where the bit is set, plus the bias gradient (column sums)
    gy = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.1).bfloat16()
    cs = torch.zeros(N, device="cuda")
    df = C.gemm(gy, w.t(), force_path=force_path, relu_bits=bits, colsum_out=cs)
    dref = torch.where(pos, gy.float() @ w.float().t(), torch.zeros(M, N, device="cuda"))
    _check(df, dref, 1e-2)
    _check(cs, df.float().sum(0), 1e-2)
    via_mask = C.gemm(gy, w.t(), force_path=force_path, relu_mask=f)
    _check(df[sure], via_mask[sure].float(), 1e-2)
    assert int(C.read_device_error(True)) == 0


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 8192), (1024, 3072, 4096), (296, 200, 1000), (512, 520, 2048)])
@pytest.mark.parametrize("pair", [1, 0])
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_gemm_tc_stream_k(M, N, K, pair, beta):
    """Stream-K (every CTA or pair takes an equal run of the tiles x k-blocks
    space and adds its pieces into the fp32 output with TMA reduces), forced
    through the tiling override, on weight-gradient layouts (both operands
    M/N-major), against the fp32 product of the same operands."""
    C = _C()
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(K, M, device="cuda", generator=g).bfloat16().t()
    b = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    acc0 = torch.randn(M, N, device="cuda", generator=g)
    out = acc0.clone()
    try:
        C.gemm_set_tiling(256, -1, pair)
        C.gemm(a, b, beta=beta, out=out, force_path=1)
    finally:
        C.gemm_set_tiling(0, 0, -1)
    ref = beta * acc0 + a.float() @ b.float()
    err = (out - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item(), f"max err {err}"
    assert int(C.read_device_error(True)) == 0


@pytest.mark.parametrize("M,N,K", [(512, 1024, 256), (8192, 1024, 512), (256, 4096, 128)])
@pytest.mark.parametrize("bias", [False, True])
def test_gemm_tc_colsum_in_registers(M, N, K, bias):
    """Column sums fused into an epilogue with no staged input (summed over
    each 32-row chunk in registers by shuffles), against the sums of the
    GEMM's own output."""
    C = _C()
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = (torch.randn(K, N, device="cuda", generator=g) * 0.1).bfloat16()
    bv = torch.randn(N, device="cuda", generator=g) if bias else None
    cs = torch.full((N,), 3.0, device="cuda")
    out = C.gemm(a, b, bias=bv, out_dtype=torch.float32, colsum_out=cs, colsum_scale=0.5, colsum_accumulate=True)
    _check(out, _ref(a, b, bv), 1e-3)
    ref = 3.0 + 0.5 * out.sum(0)
    err = (cs - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-3, f"max err {err}"
    assert int(C.read_device_error(True)) == 0


@pytest.mark.parametrize("M,N,K", [(512, 1024, 256), (264, 200, 128), (8192, 1024, 1024)])
@pytest.mark.parametrize("strided", [False, True])
def test_gemm_tc_residual_in_registers(M, N, K, strided):
    """bf16 residual added on the row-per-lane epilogue (contiguous rows read
    as 16-byte vectors, or element by element for a ragged / strided one),
    with bias and ReLU, against fp32 PyTorch."""
    C = _C()
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = (torch.randn(K, N, device="cuda", generator=g) * 0.1).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g)
    base = torch.randn(M, N + (3 if strided else 0), device="cuda", generator=g).bfloat16()
    res = base[:, :N]
    out = C.gemm(a, b, bias=bias, act=1, residual=res, force_path=1)
    ref = torch.relu(a.float() @ b.float() + bias + res.float())
    _check(out, ref, 1e-2)
    assert int(C.read_device_error(True)) == 0


@pytest.mark.parametrize("M,N,K", [(128, 47, 256), (256, 47, 2048), (32, 128, 784), (200, 10, 1000)])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_gemm_simt_split_k(M, N, K, dt):
    """Small GEMMs on the SIMT path split K across blocks (fp32 partials and a
    finish kernel): plain, bias + ReLU, and accumulate into C."""
    C = _C()
    torch.manual_seed(M + K)
    a = torch.randn(M, K, device="cuda").to(dt)
    b = torch.randn(K, N, device="cuda").to(dt)
    tol = 1e-4 if dt == torch.float32 else 1e-2
    _check(C.gemm(a, b, force_path=2), _ref(a, b), tol)
    bias = torch.randn(N, device="cuda")
    _check(C.gemm(a, b, bias=bias, act=1, force_path=2), _ref(a, b, bias, act=1), tol)
    acc = torch.randn(M, N, device="cuda")
    ref = acc + a.float() @ b.float()
    C.gemm(a, b, beta=1.0, out=acc, force_path=2)
    _check(acc, ref, 1e-4)
    torch.cuda.synchronize()
    assert C.read_device_error(True) == 0
