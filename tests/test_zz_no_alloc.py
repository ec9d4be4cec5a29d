"""mb2_block_step_static: the decode step whose workspace is the library's own
fixed device array (for callers that cannot allocate device memory).

Checked through the C ABI against mb2_block_step with a caller workspace, on
two calls in a row (the second call finds the first call's leftovers in the
shared array), and with the device's free memory unchanged across a warmed-up
call.  Named so that pytest collects it last; it also passes alone in a fresh
process, where its first call performs the per-device set-up."""
import ctypes

import pytest
import torch

from cpu_mamba_b200 import CPUMamba, _lib

STATIC_BYTES = 8 << 20
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _block(dtype, d_model=128, d_state=16, seed=0):
    torch.manual_seed(seed)
    m = CPUMamba(d_model=d_model, d_state=d_state).cuda().to(dtype)
    with torch.no_grad():
        m.dt_proj.bias.uniform_(-4.0, -2.0)
    return m


def _step_workspace(m, blk, x, h, conv):
    L = _lib.lib()
    B = x.shape[0]
    n = L.mb2_step_workspace_bytes(ctypes.byref(blk), B)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    _lib.check(L.mb2_block_step(ctypes.byref(blk), x.data_ptr(), out.data_ptr(), h.data_ptr(),
                                conv.data_ptr(), B, ws.data_ptr(), n, _lib.stream_of(x)),
               "mb2_block_step")
    return out


def _step_static_into(blk, x, out, h, conv):
    _lib.check(_lib.lib().mb2_block_step_static(ctypes.byref(blk), x.data_ptr(), out.data_ptr(),
                                                h.data_ptr(), conv.data_ptr(), x.shape[0],
                                                _lib.stream_of(x)),
               "mb2_block_step_static")


def _close(a, b, dtype):
    if dtype == torch.float32:
        return (a.float() - b.float()).abs().max().item() <= TOL[dtype]
    rel = ((a.float() - b.float()).abs() / (b.float().abs().clamp(min=1e-3) + 1e-6)).mean().item()
    return rel <= TOL[dtype]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,batch", [(torch.float32, 5), (torch.float32, 300),
                                         (torch.bfloat16, 64)])
def test_static_step_matches_workspace_step(dtype, batch):
    m = _block(dtype)
    keep = []
    blk = m._descriptor(keep)
    assert _lib.lib().mb2_step_workspace_bytes(ctypes.byref(blk), batch) <= STATIC_BYTES
    g = torch.Generator(device="cuda").manual_seed(batch)
    prompt = torch.randn(batch, 7, m.d_model, device="cuda", generator=g).to(dtype)
    _, state = m.forward_with_final_state(prompt)
    h_a, conv_a = state["h"].clone(), state["conv_state"].clone()
    h_b, conv_b = state["h"].clone(), state["conv_state"].clone()
    for i in range(2):   # two calls in a row
        x = torch.randn(batch, m.d_model, device="cuda", generator=g).to(dtype)
        y_ref = _step_workspace(m, blk, x, h_a, conv_a)
        y = torch.empty_like(x)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        _step_static_into(blk, x, y, h_b, conv_b)
        torch.cuda.synchronize()
        if i > 0:   # the first call may still load kernels lazily
            assert torch.cuda.mem_get_info()[0] == free_before, "the static step allocated"
        assert torch.isfinite(y.float()).all()
        assert _close(y, y_ref, dtype)
        assert (h_b - h_a).abs().max().item() <= 1e-5
        assert _close(conv_b, conv_a, dtype)
    assert _lib.device_status() == 0


def test_static_step_rejects_batch_beyond_array():
    """The size check comes before any CUDA call, so this runs without a GPU."""
    blk = _lib.Block()
    blk.d_model, blk.d_inner, blk.d_state, blk.d_conv, blk.dt_rank = 1024, 2048, 16, 4, 64
    blk.dtype = 0
    L = _lib.lib()
    batch = 4096
    assert L.mb2_step_workspace_bytes(ctypes.byref(blk), batch) > STATIC_BYTES
    rc = L.mb2_block_step_static(ctypes.byref(blk), None, None, None, None, batch, None)
    assert rc == 6
    assert b"fixed" in L.mb2_last_error()
