"""The allocation-free attention entry point (``mimir_fmha_fwd_noalloc``), called through its
exported C symbol exactly as a caller without access to an allocator would call it: raw device
pointers, a stream handle, and no PyTorch allocation inside the call.  Its output must match
the regular entry point (``_C.fmha_fwd``) on two consecutive calls, the second reusing the
shared scratch left behind by the first.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    import mimir_b200._C as ext_module
    lib = ctypes.CDLL(ext_module.__file__)
    fn = lib.mimir_fmha_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _close(a, b, atol, rtol, name):
    err = (a.float() - b.float()).abs()
    assert bool((err <= atol + rtol * b.float().abs()).all()), f"{name}: max abs err {err.max().item():.3e}"


@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_entry(causal):
    from mimir_b200 import ops
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    from mimir_b200.ops.attention import attention_plan

    fn = _symbol()
    torch.manual_seed(0)
    lengths, prefixes, H, KV = [700, 129, 1000], [300, 1, 0], 8, 2
    T = sum(lengths) + 21
    p = np.array(prefixes, np.int32)
    c = np.array(lengths, np.int32) - p
    tensors, _ = compute_aux_seq_tensors_scalars(p, c, T)
    cu = torch.from_numpy(tensors["cu_seqlens"]).cuda()
    pl = torch.from_numpy(tensors["prefix_lens"]).cuda()
    q = torch.randn(T, H * 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, KV * 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(T, KV * 128, device="cuda").to(torch.bfloat16)
    nseq = len(lengths)
    tiles, ntiles = attention_plan(cu, pl, nseq, T, causal, kind="fwd")  # the one-tile kernel's schedule
    ref_out, ref_lse = ops.ext().fmha_fwd(q, 0, k, 0, v, 0, None, 0, H, KV, causal, cu, pl, nseq, tiles, ntiles)
    total = sum(lengths)
    lse_ld = ref_lse.shape[1]
    out = torch.zeros(T, H * 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(H, lse_ld, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out.zero_()
        lse.zero_()
        rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), out.data_ptr(),
                lse.data_ptr(), lse_ld, cu.data_ptr(), pl.data_ptr(), nseq, T, H, KV, int(causal), stream)
        assert rc == 0, f"call {call}: error code {rc}"
        torch.cuda.synchronize()
        _close(out[:total], ref_out[:total], 2e-2, 2e-2, f"out (call {call})")
        _close(lse[:, :total], ref_lse[:, :total], 1e-3, 1e-4, f"lse (call {call})")


def test_noalloc_rejects_oversized_calls():
    fn = _symbol()
    big = 16384 * 128 + 1  # more tiles than the fixed scratch holds
    x = torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16)
    cu = torch.zeros(2, device="cuda", dtype=torch.int32)
    lse = torch.zeros(1, 8, device="cuda")
    rc = fn(x.data_ptr(), 128, x.data_ptr(), 128, x.data_ptr(), 128, x.data_ptr(), lse.data_ptr(), big,
            cu.data_ptr(), cu.data_ptr(), 1, big, 1, 1, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == -2
