"""The tcgen05 CTA-pair dense GEMM (``csrc/gemm.cu``) against plain PyTorch fp32 matmuls.

bf16 operands, fp32 accumulation, bf16 (or fp32) output: the error bound is relative to the
largest reference magnitude, like the other kernel tests.
"""
import threading

import pytest
import torch
import torch.nn.functional as F

from mimir_b200 import ops
from mimir_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _close(a, b, tol=1.5e-2, name=""):
    a, b = a.float(), b.float()
    scale = b.abs().max().item() + 1e-6
    err = ((a - b).abs() / scale).max().item()
    assert err <= tol, f"{name}: max error {err:.3e} of the largest magnitude {scale:.3e}"


def _rand(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


# (M, N, K): ragged rows, a column count that is not a multiple of the 256-wide tile, short K
SHAPES = [(1000, 352, 200), (256, 256, 64), (4096, 2048, 2048), (300, 5632, 136), (17, 64, 8)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("bn", [256, 128])
def test_forward_nt(M, N, K, bn):
    x, w = _rand(M, K, seed=1), _rand(N, K, seed=2)
    y = ops.ext().gemm(x, False, w, False, bn=bn)
    _close(y, x.float() @ w.float().t(), name=f"nt {M}x{N}x{K}")
    assert G.status(0) == 0


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_input_grad_nn(M, N, K):
    dy, w = _rand(M, K, seed=3), _rand(K, N, seed=4)
    _close(G.mm_nn(dy, w), dy.float() @ w.float(), name=f"nn {M}x{N}x{K}")
    assert G.status(0) == 0


@pytest.mark.parametrize("M,N,K", [(352, 992, 1000), (256, 256, 64), (2048, 2048, 4096), (5632, 64, 77)])
def test_weight_grad_tn(M, N, K):
    dy, x = _rand(K, M, seed=5), _rand(K, N, seed=6)
    _close(G.mm_tn(dy, x), dy.float().t() @ x.float(), name=f"tn {M}x{N}x{K}")
    assert G.status(0) == 0


@pytest.mark.parametrize("name,n_out,n_in", [("gqkv", 5120, 2048), ("o", 2048, 2048), ("gate_up", 11264, 2048),
                                              ("down", 2048, 5632), ("lm_head", 65536, 2048)])
def test_model_projection_shapes(name, n_out, n_in):
    """The five projections of the 1.3B bench model, all three GEMMs, 4096 tokens."""
    T = 4096
    x, w, dy = _rand(T, n_in, seed=7), _rand(n_out, n_in, seed=8, scale=n_in ** -0.5), _rand(T, n_out, seed=9)
    xf, wf, dyf = x.float(), w.float(), dy.float()
    _close(G.mm_nt(x, w), xf @ wf.t(), name=f"{name} forward")
    _close(G.mm_nn(dy, w), dyf @ wf, name=f"{name} input grad")
    _close(G.mm_tn(dy, x), dyf.t() @ xf, name=f"{name} weight grad")
    assert G.status(0) == 0


def test_fp32_output_and_in_place_accumulation():
    M, N, K = 512, 768, 384
    dy, x = _rand(K, M, seed=10), _rand(K, N, seed=11)
    acc32 = torch.randn(M, N, device="cuda")
    ref32 = acc32 + dy.float().t() @ x.float()
    G.mm_tn(dy, x, out=acc32, accumulate=True)
    _close(acc32, ref32, 1e-4, "fp32 accumulate")
    acc16 = _rand(M, N, seed=12)
    ref16 = acc16.float() + dy.float().t() @ x.float()
    G.mm_tn(dy, x, out=acc16, accumulate=True)
    _close(acc16, ref16, 1.5e-2, "bf16 accumulate")
    a, b = _rand(M, K, seed=13), _rand(N, K, seed=14)
    add = _rand(M, N, seed=15)
    y = ops.ext().gemm(a, False, b, False, None, add, 0.5, -2.0)
    _close(y, 0.5 * (a.float() @ b.float().t()) - 2.0 * add.float(), name="alpha/beta epilogue")
    assert G.status(0) == 0


@pytest.mark.parametrize("T,D,F_", [(1000, 256, 384), (4096, 2048, 5632)])
def test_swiglu_epilogues(T, D, F_):
    x, w_gu, w_dn = _rand(T, D, seed=16), _rand(2 * F_, D, seed=17, scale=D ** -0.5), _rand(D, F_, seed=18,
                                                                                             scale=F_ ** -0.5)
    h, gu = ops.ext().gemm_swiglu(x, w_gu)
    gu_ref = (x.float() @ w_gu.float().t())
    _close(gu, gu_ref, name="gate|up")
    assert torch.equal(h, ops.ext().swiglu_fwd(gu)), "fused product differs from the SwiGLU kernel on the same gate|up"
    dy = _rand(T, D, seed=19)
    dgu = ops.ext().gemm_swiglu_bwd(dy, w_dn, gu)
    dh_ref = (dy.float() @ w_dn.float()).to(torch.bfloat16)
    _close(dgu, ops.ext().swiglu_bwd(dh_ref, gu), 2e-2, "fused SwiGLU backward")
    assert G.status(0) == 0


def test_linear_and_mlp_autograd_match_fp32():
    torch.manual_seed(0)
    T, D, F_ = 777, 512, 1408
    x = _rand(T, D, seed=20).requires_grad_(True)
    w_gu = _rand(2 * F_, D, seed=21, scale=D ** -0.5).requires_grad_(True)
    w_dn = _rand(D, F_, seed=22, scale=F_ ** -0.5).requires_grad_(True)
    assert G.swiglu_mlp_supported(x, w_gu, w_dn)
    y = ops.swiglu_mlp(x, w_gu, w_dn)
    xf, guf, dnf = (t.detach().float().requires_grad_(True) for t in (x, w_gu, w_dn))
    g, u = (xf @ guf.t()).chunk(2, dim=-1)
    yr = (F.silu(g) * u) @ dnf.t()
    _close(y, yr, 2e-2, "mlp forward")
    dy = _rand(T, D, seed=23)
    y.backward(dy)
    yr.backward(dy.float())
    for name, a, b in (("dx", x.grad, xf.grad), ("dw_gu", w_gu.grad, guf.grad), ("dw_down", w_dn.grad, dnf.grad)):
        _close(a, b, 3e-2, f"mlp {name}")
    w = _rand(384, D, seed=24).requires_grad_(True)
    x2 = _rand(T, D, seed=25).requires_grad_(True)
    y2 = ops.linear(x2, w)
    y2r = x2.detach().float() @ w.detach().float().t()
    _close(y2, y2r, name="linear forward")
    d2 = _rand(T, 384, seed=26)
    y2.backward(d2)
    _close(x2.grad, d2.float() @ w.detach().float(), name="linear dx")
    _close(w.grad, d2.float().t() @ x2.detach().float(), name="linear dw")
    assert G.status(0) == 0


def test_first_call_on_a_fresh_host_thread():
    """A host thread that has made no CUDA call yet (like the autograd engine's worker) has no
    current context; the TMA descriptors must still be built (the op binds the primary context)."""
    x, w = _rand(777, 512, seed=29), _rand(1408, 512, seed=30)
    result = {}

    def work():
        try:
            result["y"] = G.mm_nt(x, w)
            torch.cuda.synchronize()
        except Exception as exc:  # noqa: BLE001 - reported below
            result["error"] = exc

    t = threading.Thread(target=work)
    t.start()
    t.join()
    assert "error" not in result, result.get("error")
    _close(result["y"], x.float() @ w.float().t(), name="fresh thread")


def test_bounded_wait_times_out_and_the_next_launch_is_clean():
    """The test hook withholds one accumulator release, so the MMA issuer's wait (limit 2 ms)
    runs out: the kernel must return with a timeout status instead of hanging (5: the MMA issuer's
    accumulator wait; the producer's stage wait (6) or the epilogue's wait (3) may report first
    within the polling granularity), and the next normal launch on the same GPU must be correct
    with status 0."""
    x, w = _rand(16384, 512, seed=27), _rand(2048, 512, seed=28)  # 512 tiles: several per CTA pair
    ops.ext().gemm(x, False, w, False, wait_ns=2_000_000, inject=1)
    torch.cuda.synchronize()
    from mimir_b200.ops._ext import KernelTimeout, check_kernel_status, kernel_status
    codes = kernel_status(torch.device("cuda", 0))  # reads and clears, like the training loop
    assert codes["gemm"] in (3, 5, 6) and codes["attention"] == 0 and codes["grouped_gemm"] == 0
    ops.ext().gemm(x, False, w, False, wait_ns=2_000_000, inject=1)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeout):
        check_kernel_status(torch.device("cuda", 0), step=7)
    _close(G.mm_nt(x, w), x.float() @ w.float().t(), name="after the timeout")
    assert G.status(0) == 0


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_batched_problems_match_per_problem_matmuls(a_mn, b_mn):
    """A batch of independent problems (3-D operands) in one launch, with the alpha/beta epilogue."""
    B, M, N, K = 3, 384, 352, 320
    a = _rand(B, K, M, seed=31) if a_mn else _rand(B, M, K, seed=31)
    b = _rand(B, K, N, seed=32) if b_mn else _rand(B, N, K, seed=32)
    add = _rand(B, M, N, seed=33)
    out = ops.ext().gemm(a, a_mn, b, b_mn, None, add, 0.75, 0.5)
    af = a.float().mT if a_mn else a.float()
    bf = b.float() if b_mn else b.float().mT
    for i in range(B):
        _close(out[i], 0.75 * (af[i] @ bf[i]) + 0.5 * add[i].float(), name=f"batch {i}")
    assert G.status(0) == 0
