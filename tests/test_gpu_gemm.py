"""The tcgen05 tensor-core GEMM (csrc/gemm_tc.cu) against float64 references.

fp32 mode (3-term TF32 split) must be as accurate as an fp32 FMA GEMM: error
within a small multiple of the CUDA-core kernel's own error against float64.
bf16 mode: bf16 operands, fp32 accumulation, bf16 output rounding only."""
import pytest
import torch

from cpu_mamba_b200 import _lib, ops

pytestmark = pytest.mark.gpu

SHAPES = [(256, 128, 32), (1000, 200, 100), (300, 96, 1536), (4096, 3072, 768), (2049, 768, 1536)]


def _data(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    w = (torch.rand(N, K, generator=g) * 2 - 1) / K ** 0.5
    b = torch.randn(N, generator=g) * 0.1
    return x, w, b


@pytest.mark.parametrize("shape", SHAPES)
def test_tf32x3_matches_float64(shape):
    M, N, K = shape
    x, w, b = _data(M, N, K, sum(shape))
    ref = (x.double() @ w.double().T + b.double()).float()
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    y_tc = ops.linear(xd, wd, bd, weight_split=ops.split_tf32(wd)).cpu()
    y_fma = ops.linear(xd, wd, bd).cpu()
    assert _lib.device_status() == 0
    e_tc = (y_tc - ref).abs().max().item()
    e_fma = (y_fma - ref).abs().max().item()
    assert e_tc <= max(4 * e_fma, 2e-6), (e_tc, e_fma)


@pytest.mark.parametrize("shape", SHAPES)
def test_bf16_matches_float64_of_rounded_operands(shape):
    M, N, K = shape
    x, w, b = _data(M, N, K, 7 + sum(shape))
    xb, wb, bb = x.bfloat16(), w.bfloat16(), b.bfloat16()
    ref = xb.double() @ wb.double().T + bb.double()
    y = ops.linear(xb.cuda(), wb.cuda(), bb.cuda()).cpu().double()
    assert _lib.device_status() == 0
    # only the final bf16 rounding (2^-9 relative) plus fp32 accumulation noise
    err = ((y - ref).abs() / (ref.abs() + 1e-2)).max().item()
    assert err <= 2 ** -8, err


def test_split_tf32_is_exact_decomposition():
    w = torch.randn(37, 53, device="cuda")
    s = ops.split_tf32(w)
    hi, lo = s[0], s[1]
    bits = lambda t: t.view(torch.int32) & 0x1FFF
    assert (bits(hi) == 0).all() and (bits(lo) == 0).all()      # TF32-representable
    assert ((hi.double() + lo.double() - w.double()).abs() <= w.double().abs() * 2 ** -21).all()


def test_column_remap_and_strided_output():
    """x_proj-style launch: three output segments written at aligned offsets."""
    M, K, R, S = 512, 256, 12, 16
    x, w, _ = _data(M, R + 2 * S, K, 3)
    xd, wd = x.cuda(), w.cuda()
    ref = ops.linear(xd, wd, None, weight_split=ops.split_tf32(wd))
    blk = _lib.lib()
    ldy = 16 + 16 + 16
    y = torch.full((M, ldy), float("nan"), device="cuda")
    split = ops.split_tf32(wd)
    # direct C-ABI call through the internal remap is exercised by the block
    # forward; here check the plain strided store path (ld_y > N)
    _lib.check(blk.mb2_linear(0, xd.data_ptr(), K, wd.data_ptr(), split.data_ptr(), None,
                              y.data_ptr(), ldy, M, R + 2 * S, K, 0, _lib.stream_of(xd)), "linear")
    assert torch.equal(y[:, :R + 2 * S], ref)
    assert torch.isnan(y[:, R + 2 * S:]).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M", [64, 2048])
def test_softplus_epilogue(dtype, M):
    """dt_proj's GEMM applies F.softplus (beta 1, threshold 20) to the stored value."""
    N, K = 768, 48
    x, w, b = _data(M, N, K, 5)
    x = x * 6                                  # reach both softplus branches (|v| > 20)
    xd, wd, bd = x.to(dtype).cuda(), w.to(dtype).cuda(), b.to(dtype).cuda()
    split = ops.split_tf32(wd) if dtype == torch.float32 else None
    y = ops.linear(xd, wd, bd, weight_split=split, softplus=True).cpu()
    lin = ops.linear(xd, wd, bd, weight_split=split).cpu()
    ref = torch.nn.functional.softplus(lin.float())
    if dtype == torch.float32:
        assert (y - ref).abs().max().item() <= 2e-6
    else:
        assert ((y.float() - ref).abs() / (ref.abs() + 1e-3)).max().item() <= 2 ** -8


# ------------------------------------------------------------------ F16X3 ---
F16_SHAPES = [(256, 128, 64), (1000, 200, 104), (300, 96, 1536), (4096, 3072, 768),
              (2049, 768, 1536), (1024, 128, 3072), (4096, 3072, 1536)]


def _f32_err(x, w, b, ref):
    """The float32 CPU GEMM's own distance to float64 (the yardstick)."""
    return ((x @ w.T + b).double() - ref).abs().max().item()


@pytest.mark.parametrize("shape", F16_SHAPES)
@pytest.mark.parametrize("mag", [1.0, 3e3, 1e-4])
def test_f16x3_matches_float64(shape, mag):
    """The fp16-split GEMM as accurate as an fp32 GEMM at every K (the segment
    drains bound the tensor core's truncation), whatever the operands' scale."""
    M, N, K = shape
    x, w, b = _data(M, N, K, 11 + sum(shape))
    x = x * mag
    w[0, :8] *= 40.0                        # a few outliers, as quantised weights have
    ref = x.double() @ w.double().T + b.double()
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    y = ops.linear(xd, wd, bd, weight_f16=ops.split_f16(wd)).cpu()
    assert _lib.device_status() == 0
    e = (y.double() - ref).abs().max().item()
    e_cpu = _f32_err(x, w, b, ref)
    scale = ref.abs().max().item()
    assert e <= max(3 * e_cpu, 2e-7 * scale), (e, e_cpu, scale)


def test_f16x3_large_k_beats_tf32x3():
    """K = 3072 at large magnitudes (config 3's x_proj / out_proj): the segment
    drains keep the error at the fp32 GEMM's level, where the 3xTF32 kernel's
    single accumulation over K drifts."""
    M, N, K = 2048, 768, 3072
    x, w, b = _data(M, N, K, 21)
    x = x * 30
    ref = x.double() @ w.double().T + b.double()
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    e16 = (ops.linear(xd, wd, bd, weight_f16=ops.split_f16(wd)).cpu().double() - ref).abs().max().item()
    e_cpu = _f32_err(x, w, b, ref)
    assert e16 <= 3 * e_cpu, (e16, e_cpu)


def test_f16x3_zero_and_tail_shapes():
    """All-zero x (scale 1), M not a multiple of 128, N not of 128."""
    M, N, K = 777, 40, 64
    x, w, b = _data(M, N, K, 3)
    wd = w.cuda()
    y = ops.linear(torch.zeros(M, K, device="cuda"), wd, b.cuda(), weight_f16=ops.split_f16(wd))
    assert torch.equal(y.cpu(), b.expand(M, N))
    y = ops.linear(x.cuda(), wd, None, weight_f16=ops.split_f16(wd)).cpu()
    ref = x.double() @ w.double().T
    assert (y.double() - ref).abs().max().item() <= 3 * _f32_err(x, w, torch.zeros(N), ref) + 1e-7


def test_split_f16_layout():
    """Header (2^-e scale), hi and lo planes: w * 2^e == hi + lo to 2^-22."""
    w = torch.randn(37, 64, device="cuda") * 0.01
    buf = ops.split_f16(w)
    inv = buf[:4].view(torch.float32).item()
    n = w.numel()
    planes = buf[4096:4096 + 4 * n].view(torch.float16)
    hi, lo = planes[:n].view(37, 64), planes[n:].view(37, 64)
    scaled = w.double() / inv
    assert 2 ** 14 <= scaled.abs().max().item() < 2 ** 15
    err = (hi.double() + lo.double() - scaled).abs()
    assert (err <= scaled.abs() * 2 ** -21 + 2 ** -24).all()


@pytest.mark.parametrize("M", [300, 2048])
def test_f16x3_softplus_epilogue(M):
    N, K = 768, 64
    x, w, b = _data(M, N, K, 5)
    x = x * 6
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    s16 = ops.split_f16(wd)
    y = ops.linear(xd, wd, bd, weight_f16=s16, softplus=True).cpu()
    lin = ops.linear(xd, wd, bd, weight_f16=s16).cpu()
    assert (y - torch.nn.functional.softplus(lin)).abs().max().item() <= 2e-6


@pytest.mark.parametrize("shape", [(4096, 3072, 768), (2049, 768, 1536), (1000, 300, 104),
                                   (300, 256, 3072), (27180, 512, 40)])
@pytest.mark.parametrize("scale", [1e-4, 1.0, 3e3])
def test_f16x3_wide_tiles(shape, scale):
    """128 x 256 tiles (the default for N >= 256: 256-wide MMAs, x's split in
    shared memory) against 128 x 128 tiles and float64: the same segment sums
    of the same products, within 3x of an fp32 CPU GEMM's own error."""
    M, N, K = shape
    x, w, b = _data(M, N, K, 7 + sum(shape))
    x = x * scale
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    s16 = ops.split_f16(wd)
    y_wide = ops.linear(xd, wd, bd, weight_f16=s16)
    y_narrow = ops.linear(xd, wd, bd, weight_f16=s16, sm_pair=0)
    assert _lib.device_status() == 0
    ref = x.double() @ w.double().T + b.double()
    bound = 3 * _f32_err(x, w, b, ref) + 1e-7 * scale
    err_w = (y_wide.cpu().double() - ref).abs().max().item()
    err_n = (y_narrow.cpu().double() - ref).abs().max().item()
    assert err_w <= bound, (err_w, err_n, bound)


@pytest.mark.parametrize("shape", [(4096, 3072, 768), (300, 96, 1536), (1000, 200, 104),
                                   (2049, 768, 1536), (256, 128, 64)])
def test_f16x3_sm_pairs_equal_single_sms(shape):
    """256-row tiles on pairs of SMs (cta_group::2, each SM loading half of
    W's tile) and 128-row tiles on single SMs: identical results (the same
    MMAs and the same segment sums, only the tile layout differs)."""
    M, N, K = shape
    x, w, b = _data(M, N, K, 31 + sum(shape))
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    s16 = ops.split_f16(wd)
    y1 = ops.linear(xd, wd, bd, weight_f16=s16, sm_pair=0)
    y2 = ops.linear(xd, wd, bd, weight_f16=s16, sm_pair=1)
    assert _lib.device_status() == 0
    assert torch.equal(y1, y2)
    ref = x.double() @ w.double().T + b.double()
    assert (y2.cpu().double() - ref).abs().max().item() <= 3 * _f32_err(x, w, b, ref) + 1e-7
