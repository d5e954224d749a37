"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op.
These tests require the native extension on a GPU: on a CUDA box a missing extension fails
(there is no silent fallback)."""
import pytest
import torch
import torch.nn.functional as F

from femtotron_b200.ops import matmul as G
from femtotron_b200.ops import kernels as K
from femtotron_b200.ops.ext import check_kernel_errors, native

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True, scope="module")
def _ext():
    native()  # fail loudly if the extension is missing on a GPU box
    yield
    check_kernel_errors()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (4096, 1024, 512),
                                   (300, 136, 200), (1000, 2048, 1024), (64, 8, 64)])
def test_gemm_forward(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    G.gemm(a, b, out)
    ref = a.float() @ b.float().t()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (4096, 640, 1024), (200, 72, 136)])
def test_gemm_dgrad_mn_major_b(M, N, K):
    torch.manual_seed(1)
    dy = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)      # [M, N_out] with N_out=K here
    w = torch.randn(K, N, device=DEV, dtype=torch.bfloat16)       # [N_out, K_in]
    out = G.linear_dgrad(dy, w)
    ref = dy.float() @ w.float()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("T,N,K", [(512, 256, 384), (4096, 1024, 640), (136, 200, 72)])
def test_gemm_wgrad_both_mn_major(T, N, K):
    torch.manual_seed(2)
    dy = torch.randn(T, N, device=DEV, dtype=torch.bfloat16)
    x = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    dw = torch.zeros(N, K, device=DEV, dtype=torch.float32)
    G.linear_wgrad(dy, x, dw, accumulate=False)
    ref = dy.float().t() @ x.float()
    assert rel_err(dw, ref) < 1e-2
    G.linear_wgrad(dy, x, dw, accumulate=True)
    assert rel_err(dw, 2 * ref) < 1e-2
    dwb = torch.zeros(N, K, device=DEV, dtype=torch.bfloat16)
    G.linear_wgrad(dy, x, dwb, accumulate=True)
    assert rel_err(dwb, ref) < 1e-2


def test_gemm_residual_and_mn_major_a():
    torch.manual_seed(3)
    M, N, K = 384, 512, 256
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    r = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    out = G.linear_fwd(a, b, residual=r)
    assert rel_err(out, a.float() @ b.float().t() + r.float()) < 1e-2
    at = a.t().contiguous()   # [K, M]
    out2 = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    G.gemm(at, b, out2, a_mn=True)
    assert rel_err(out2, a.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("T,F_,H", [(256, 256, 128), (1024, 688, 256), (4096, 1792, 1024)])
def test_gemm_swiglu_epilogue(T, F_, H):
    torch.manual_seed(4)
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16) * 0.5
    w = torch.randn(2 * F_, H, device=DEV, dtype=torch.bfloat16) * 0.05
    h = torch.empty(T, F_, device=DEV, dtype=torch.bfloat16)
    gu = torch.empty(T, 2 * F_, device=DEV, dtype=torch.bfloat16)
    G.gemm(x, w, h, mode="swiglu", gu=gu, gate_up_off=F_)
    g = x.float() @ w[:F_].float().t()
    u = x.float() @ w[F_:].float().t()
    assert rel_err(gu[:, :F_], g) < 1e-2 and rel_err(gu[:, F_:], u) < 1e-2
    assert rel_err(h, F.silu(g) * u) < 2e-2


def test_gemm_large_k_and_many_tiles():
    torch.manual_seed(5)
    M, N, K = 2048, 3072, 4096
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    out = G.linear_fwd(a, b)
    assert rel_err(out, a.float() @ b.float().t()) < 1e-2
    # repeat to exercise the persistent scheduler across launches
    for _ in range(3):
        out2 = G.linear_fwd(a, b)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("T,H", [(64, 256), (1000, 4096), (17, 5120), (9, 12288)])
def test_rmsnorm(T, H):
    torch.manual_seed(6)
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    y, rstd = K.rmsnorm_fwd(x, w, 1e-5)
    yr, rr = K.rmsnorm_fwd(x.cpu(), w.cpu(), 1e-5)
    assert rel_err(y.cpu(), yr) < 1e-2 and rel_err(rstd.cpu(), rr) < 1e-4
    dy = torch.randn_like(x)
    dx, dw = K.rmsnorm_bwd(dy, x, w, rstd)
    dxr, dwr = K.rmsnorm_bwd(dy.cpu(), x.cpu(), w.cpu(), rr)
    assert rel_err(dx.cpu(), dxr) < 1e-2 and rel_err(dw.cpu(), dwr) < 1e-3


def test_rope_roundtrip_and_reference():
    torch.manual_seed(7)
    B, S, nh, d = 2, 128, 6, 128
    cos, sin = K.rope_tables(d, 256, 5e5, DEV)
    x = torch.randn(B * S, nh * d + 64, device=DEV, dtype=torch.bfloat16)
    y = K.rope_(x.clone(), cos, sin, nh, d, S)
    yr = K.rope_(x.cpu().clone(), cos.cpu(), sin.cpu(), nh, d, S)
    assert rel_err(y.cpu(), yr) < 1e-2
    assert torch.equal(y[:, nh * d:], x[:, nh * d:])
    back = K.rope_(y.clone(), cos, sin, nh, d, S, inverse=True)
    assert rel_err(back, x) < 2e-2


def test_swiglu_kernels():
    torch.manual_seed(8)
    T, F_ = 333, 688
    gu = torch.randn(T, 2 * F_, device=DEV, dtype=torch.bfloat16)
    h = K.swiglu_fwd(gu, F_)
    assert rel_err(h.cpu(), K.swiglu_fwd(gu.cpu(), F_)) < 1e-2
    dh = torch.randn(T, F_, device=DEV, dtype=torch.bfloat16)
    d = K.swiglu_bwd(dh, gu, F_)
    assert rel_err(d.cpu(), K.swiglu_bwd(dh.cpu(), gu.cpu(), F_)) < 1e-2


def test_embedding_kernels():
    torch.manual_seed(9)
    V, H, T = 1000, 256, 777
    table = torch.randn(V, H, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, 2 * V, (T,), device=DEV)
    out = K.embed_fwd(ids, table, V // 2)
    assert torch.equal(out.cpu(), K.embed_fwd(ids.cpu(), table.cpu(), V // 2))
    dout = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    dt = K.embed_bwd(ids, dout, V, V // 2)
    assert rel_err(dt.cpu(), K.embed_bwd(ids.cpu(), dout.cpu(), V, V // 2)) < 1e-5


@pytest.mark.parametrize("T,V", [(128, 2048), (257, 32000)])
def test_cross_entropy_kernels(T, V):
    torch.manual_seed(10)
    logits = (3 * torch.randn(T, V, device=DEV)).to(torch.bfloat16)
    labels = torch.randint(0, V, (T,), device=DEV)
    labels[::7] = -100
    st = K.xent_stats(logits, labels, 0)
    lse = st[:, 0] + torch.log(st[:, 1])
    ref = torch.logsumexp(logits.float(), -1)
    assert (lse - ref).abs().max().item() < 1e-3
    scale = torch.tensor([0.5], device=DEV)
    d = K.xent_bwd_(logits.clone(), labels, lse, scale, 0)
    x = logits.float().requires_grad_(True)
    F.cross_entropy(x, labels, ignore_index=-100, reduction="sum").mul(0.5).backward()
    assert rel_err(d, x.grad) < 1e-2


def test_adamw_matches_torch():
    torch.manual_seed(11)
    shapes = [(1000,), (64, 300), (70001,)]
    ps = [torch.randn(s, device=DEV) for s in shapes]
    gs = [torch.randn(s, device=DEV).to(torch.bfloat16) for s in shapes]
    ref_p = [p.clone().requires_grad_(True) for p in ps]
    opt = torch.optim.AdamW(ref_p, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    ms = [torch.zeros_like(p) for p in ps]
    vs = [torch.zeros_like(p) for p in ps]
    outs = [torch.empty(s, device=DEV, dtype=torch.bfloat16) for s in shapes]
    for step in range(1, 4):
        for rp, g in zip(ref_p, gs):
            rp.grad = g.float()
        opt.step()
        K.adamw_multi(ps, ms, vs, gs, outs, [0.1] * 3, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, step=step)
    for p, rp, o in zip(ps, ref_p, outs):
        assert rel_err(p, rp.detach()) < 1e-5
        assert rel_err(o, rp.detach()) < 1e-2


def test_adamw_fp32_grads_and_unaligned_views():
    """fp32 gradients, and parameter / state views that start 4 bytes past a 16-byte boundary
    (element-wise path) next to aligned ones (16-byte vector path)."""
    torch.manual_seed(12)
    base = [torch.randn(5003, device=DEV) for _ in range(3)]
    ps = [base[0][1:2001], base[0][2004:5003], torch.randn(4099, device=DEV)]
    ms = [torch.zeros(2001, device=DEV)[1:], torch.zeros(2999, device=DEV), torch.zeros(4099, device=DEV)]
    vs = [torch.zeros(2001, device=DEV)[1:], torch.zeros(2999, device=DEV), torch.zeros(4099, device=DEV)]
    gs = [torch.randn(p.numel(), device=DEV) for p in ps]
    ref_p = [p.clone().requires_grad_(True) for p in ps]
    opt = torch.optim.AdamW(ref_p, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        for rp, g in zip(ref_p, gs):
            rp.grad = g
        opt.step()
        K.adamw_multi(ps, ms, vs, gs, [], [0.1] * 3, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, step=step)
    for p, rp in zip(ps, ref_p):
        assert rel_err(p, rp.detach()) < 1e-5


def test_sumsq_multi():
    ts = [torch.randn(1000, device=DEV), torch.randn(3, 77, device=DEV).to(torch.bfloat16)]
    out = torch.zeros(2, device=DEV)
    K.sumsq_multi(ts, [0, 1], out)
    assert abs(out[0].item() - ts[0].pow(2).sum().item()) < 1e-2
    assert abs(out[1].item() - ts[1].float().pow(2).sum().item()) < 1e-2
