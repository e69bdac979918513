"""The allocation-free attention entry point (``mimir_fmha_fwd_noalloc``).

It is called here through its exported C symbol, the way a caller that cannot allocate device
memory calls it (an inference runtime or plugin that owns all device memory, or code under a
fixed memory budget): raw device pointers, a stream handle, and no allocation inside the call.
Its output must match the regular entry point (``_C.fmha_fwd``) and the fp32 dense oracle on
two consecutive calls, the second reusing the shared scratch left behind by the first, and the
kernel status read through ``mimir_fmha_noalloc_status`` must be 0 after each call.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch


def _lib():
    import mimir_b200._C as ext_module
    return ctypes.CDLL(ext_module.__file__)


def _symbol():
    fn = _lib().mimir_fmha_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _status_fn():
    fn = _lib().mimir_fmha_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return fn


def _read_status(stream) -> int:
    value = ctypes.c_int(-99)
    rc = _status_fn()(stream, ctypes.byref(value))
    assert rc == 0, f"status readout failed with {rc}"
    return value.value


def _close(a, b, atol, rtol, name):
    err = (a.float() - b.float()).abs()
    assert bool((err <= atol + rtol * b.float().abs()).all()), f"{name}: max abs err {err.max().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_entry_and_oracle(causal):
    from mimir_b200 import ops
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    from mimir_b200.ops.attention import attention_plan

    fn = _symbol()
    torch.manual_seed(0)
    lengths, prefixes, H, KV = [700, 129, 1000], [300, 1, 0], 8, 2
    T = sum(lengths) + 21
    p = np.array(prefixes, np.int32)
    c = np.array(lengths, np.int32) - p
    tensors, scalars = compute_aux_seq_tensors_scalars(p, c, T)
    meta = {k: torch.from_numpy(v).cuda() for k, v in tensors.items()} | scalars
    cu, pl = meta["cu_seqlens"], meta["prefix_lens"]
    q = torch.randn(T, H * 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, KV * 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(T, KV * 128, device="cuda").to(torch.bfloat16)
    nseq = len(lengths)
    total = sum(lengths)
    tiles, ntiles = attention_plan(cu, pl, nseq, T, causal, kind="fwd")  # the one-tile kernel's schedule
    ref_out, ref_lse = ops.ext().fmha_fwd(q, 0, k, 0, v, 0, None, 0, H, KV, causal, cu, pl, nseq, tiles, ntiles)
    oracle = ops.dense_prefixlm_attention(q.view(T, H, 128).float(), k.view(T, KV, 128).float(),
                                          v.view(T, KV, 128).float(), causal, **meta).view(T, H * 128)
    lse_ld = ref_lse.shape[1]
    out = torch.zeros(T, H * 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(H, lse_ld, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out.fill_(float("nan"))
        lse.fill_(float("nan"))
        rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), out.data_ptr(),
                lse.data_ptr(), lse_ld, cu.data_ptr(), pl.data_ptr(), nseq, T, H, KV, int(causal), stream)
        assert rc == 0, f"call {call}: error code {rc}"
        assert _read_status(stream) == 0, f"call {call}: a bounded wait inside the kernel gave up"
        _close(out[:total], ref_out[:total], 2e-2, 2e-2, f"out vs regular entry (call {call})")
        _close(lse[:, :total], ref_lse[:, :total], 1e-3, 1e-4, f"lse vs regular entry (call {call})")
        _close(out[:total], oracle[:total], 2e-2, 2e-2, f"out vs fp32 oracle (call {call})")


@pytest.mark.gpu
def test_noalloc_rejects_oversized_calls():
    fn = _symbol()
    big = 16384 * 128 + 1  # more tiles than the fixed scratch holds
    x = torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16)
    cu = torch.zeros(2, device="cuda", dtype=torch.int32)
    lse = torch.zeros(1, 8, device="cuda")
    rc = fn(x.data_ptr(), 128, x.data_ptr(), 128, x.data_ptr(), 128, x.data_ptr(), lse.data_ptr(), big,
            cu.data_ptr(), cu.data_ptr(), 1, big, 1, 1, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == -2


def _built() -> bool:
    try:
        import mimir_b200._C  # noqa: F401
        return True
    except ImportError:
        return False


@pytest.mark.skipif(not _built(), reason="extension not built")
def test_noalloc_rejects_misaligned_output_on_the_host():
    """Argument checks run before any CUDA call, so this needs no GPU: an output pointer that is
    not 16-byte aligned (the kernel stores 16-byte vectors) and a misaligned LSE pointer are
    rejected with MIMIR_NOALLOC_ERR_ARGS."""
    fn = _symbol()
    aligned = 1 << 20  # never dereferenced: the call returns before touching memory
    args = [aligned, 128, aligned, 128, aligned, 128, aligned + 8, aligned, 8, aligned, aligned, 1, 8, 1, 1, 0, None]
    assert fn(*args) == -1
    args[6], args[7] = aligned, aligned + 2
    assert fn(*args) == -1
    assert _status_fn()(None, None) == -1  # no destination for the status
