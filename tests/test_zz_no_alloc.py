"""The allocation-free GDN entry point against the workspace one.

``cevk_gdn_chunk_prefill_noalloc`` exists for callers that cannot hand the
library a workspace -- hosts whose device memory belongs to their own fixed
pool, or paths where a cudaMalloc is not allowed or would stall.  Its
scratch is a fixed device array inside the library.  This file is collected
last so that a run stopping at its first failure has already run every other
test; it also passes alone in a fresh process (the first call on the device
does the one-time address lookup).
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, T, nk, nv, dk, dv, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    Cc = 2 * nk * dk + nv * dv
    conv_out = (torch.randn(B * T, Cc, generator=g) * 0.5).to(dtype).cuda()
    ab = torch.randn(B * T, 2 * nv, generator=g).to(dtype).cuda()
    z = torch.randn(B * T, nv * dv, generator=g).to(dtype).cuda()
    a_log = (torch.rand(nv, generator=g) * 2).cuda()
    dt_bias = torch.rand(nv, generator=g).cuda()
    norm_w = (torch.rand(dv, generator=g) + 0.5).to(dtype).cuda()
    s0 = (torch.randn(1, nv, dk, dv, generator=g) * 0.1).cuda()
    return conv_out, ab, z, a_log, dt_bias, norm_w, s0


def _noalloc(lib, conv_out, ab, z, a_log, dt_bias, norm_w, s0, B, T, nk, nv, dk, dv, dt):
    y = torch.empty(B * T, nv * dv, dtype=conv_out.dtype, device="cuda")
    s_out = torch.empty(B, nv, dk, dv, device="cuda")
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.cevk_gdn_chunk_prefill_noalloc(
        p(conv_out), conv_out.shape[1], p(ab), ab.stride(0), p(z), z.stride(0), p(a_log), p(dt_bias), p(norm_w), 1e-6,
        p(s0), 0, p(s_out), p(y), B, T, nk, nv, dk, dv, dt, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.cevk_last_error().decode()
    return y, s_out


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-4)])
@pytest.mark.parametrize("B,T", [(1, 150), (3, 64)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, tol, B, T):
    from cev_b200 import ops
    from cev_b200._lib import BF16, F32, lib
    nk, nv, dk, dv = 2, 4, 64, 64
    args = _inputs(B, T, nk, nv, dk, dv, dtype, 77)
    conv_out, ab, z, a_log, dt_bias, norm_w, s0 = args
    s_ref = torch.empty(B, nv, dk, dv, device="cuda")
    ws = torch.empty(ops.gdn_workspace_size(B, T, nv, dk, dv), dtype=torch.uint8, device="cuda")
    y_ref = ops.gdn_chunk_prefill(conv_out, ab, ab.stride(0), z, z.stride(0), a_log, dt_bias, norm_w, 1e-6, s0, s_ref,
                                  B, T, nk, nv, dk, dv, ws)
    dt = BF16 if dtype == torch.bfloat16 else F32
    for _ in range(2):  # the array keeps the last call's contents: a second call must not depend on them
        y, s_out = _noalloc(lib(), *args, B, T, nk, nv, dk, dv, dt)
        torch.cuda.synchronize()
        scale = y_ref.float().abs().max().item() if dtype == torch.bfloat16 else 1.0
        assert (y.float() - y_ref.float()).abs().max().item() < tol * scale
        assert (s_out - s_ref).abs().max().item() < tol


def test_noalloc_at_the_cfg4_head_shape_takes_the_core_only_path_twice():
    """A 512-token chunk at the cfg4 GDN shape (nk 16, nv 32, dk = dv = 128,
    bf16): the tensor-core scratch does not fit the static array, so the call
    runs the kernel whose only scratch is the f32 core output (8 MiB here).
    Checked against the workspace entry point given exactly that much
    workspace (the same kernel), on two calls in a row."""
    from cev_b200 import ops
    from cev_b200._lib import BF16, lib
    B, T, nk, nv, dk, dv = 1, 512, 16, 32, 128, 128
    core_bytes = B * T * nv * dv * 4
    assert ops.gdn_workspace_size(B, T, nv, dk, dv) > (16 << 20) >= core_bytes
    args = _inputs(B, T, nk, nv, dk, dv, torch.bfloat16, 78)
    conv_out, ab, z, a_log, dt_bias, norm_w, s0 = args
    s_ref = torch.empty(B, nv, dk, dv, device="cuda")
    ws = torch.empty(core_bytes, dtype=torch.uint8, device="cuda")
    y_ref = ops.gdn_chunk_prefill(conv_out, ab, ab.stride(0), z, z.stride(0), a_log, dt_bias, norm_w, 1e-6, s0, s_ref,
                                  B, T, nk, nv, dk, dv, ws)
    for _ in range(2):
        y, s_out = _noalloc(lib(), *args, B, T, nk, nv, dk, dv, BF16)
        torch.cuda.synchronize()
        assert (y.float() - y_ref.float()).abs().max().item() <= 1e-2 * y_ref.float().abs().max().item()
        assert (s_out - s_ref).abs().max().item() < 1e-4
    assert lib().cevk_device_status() == 0


def test_noalloc_rejects_sizes_over_the_static_array():
    from cev_b200._lib import E_SHAPE, F32, lib
    l = lib()
    big_t = 1 << 16  # 64k tokens x 4 heads x 64 columns x 4 B = 64 MiB > 16 MiB
    rc = l.cevk_gdn_chunk_prefill_noalloc(C.c_void_p(1), 512, C.c_void_p(1), 8, C.c_void_p(1), 256, C.c_void_p(1),
                                          C.c_void_p(1), C.c_void_p(1), 1e-6, None, 0, None, C.c_void_p(1), 1, big_t,
                                          2, 4, 64, 64, F32, None)
    assert rc == E_SHAPE
    assert "static array" in l.cevk_last_error().decode()
