"""One-GPU numerics of the fused-communication building blocks, against plain PyTorch fp32:

  * the GEMM operand gate of the fused all-gather -> GEMM (A rows and B rows), with the
    gated rows written and their flags released by another stream about 10 ms later;
  * the scatter epilogue of the GEMM (rows stored into their owner's buffer);
  * the pull kernels of the tensor-parallel collectives: ``ag_pull`` (peer chunks gathered in
    ring order, per-chunk counters that a gated GEMM consumes while the pull runs) and
    ``rs_pull`` (an owner sums its rows of every rank's partial, plus the residual);
  * the fused ZeRO reduce-scatter + fp32 cast/scale + AdamW kernel (``rs_adamw``) against
    the mean of the sources and ``torch.optim.AdamW``;
  * bounded waits: a flag that nothing sets ends the wait with an error code after its time
    limit (KernelTimeoutError on the host), the context stays usable, and the host-side
    bounded event wait raises instead of blocking.

Peers are emulated on one GPU: their buffers are local tensors and their flags are words that
a stream writes, so every wait here can be satisfied or time out without a second process."""
import pytest
import torch

from femtotron_b200.ops.ext import KernelTimeoutError, check_kernel_errors, error_flag, native
from femtotron_b200.parallel.tensor_parallel.fused import fused_gemm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _clean():
    native()
    check_kernel_errors(torch.device(DEV, 0))
    yield
    torch.cuda.synchronize()
    check_kernel_errors(torch.device(DEV, 0))


def _release_later(src, dst, flags, epoch, stream, delay_cycles=20_000_000):
    """On `stream`: sleep, copy src into dst, then write epoch into every flag.  Enqueued
    before the gated GEMM, so even if the two streams shared a hardware queue the release
    would not sit behind the GEMM that waits for it."""
    C = native()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(delay_cycles)
        dst.copy_(src)
        for i in range(flags.numel()):
            C.stream_write(flags.data_ptr() + 4 * i, epoch)


@pytest.mark.parametrize("M,N,K,chunks", [(1024, 512, 768, 4), (2048, 1024, 512, 8), (384, 256, 256, 3)])
def test_gate_a_rows_waits_for_late_chunks(M, N, K, chunks):
    torch.manual_seed(0)
    a_src = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    a = torch.zeros_like(a_src)
    flags = torch.zeros(chunks, dtype=torch.int32, device=DEV)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    rows = M // chunks
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    gate = dict(gate_flags=flags.data_ptr(), gate_op=1, gate_epoch=5, gate_off=0,
                gate_row_elems=K, gate_chunk_elems=rows * K)
    _release_later(a_src, a, flags, 5, side)  # operand arrives ~10 ms later
    fused_gemm(a, b, out, gate=gate)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert rel_err(out, a_src.float() @ b.float().t()) < 1e-2


@pytest.mark.parametrize("M,N,K,chunks", [(1024, 1024, 512, 4), (512, 768, 1024, 6)])
def test_gate_b_rows_waits_for_late_chunks(M, N, K, chunks):
    torch.manual_seed(1)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b_src = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros_like(b_src)
    flags = torch.zeros(chunks, dtype=torch.int32, device=DEV)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    gate = dict(gate_flags=flags.data_ptr(), gate_op=2, gate_epoch=2, gate_off=0,
                gate_row_elems=K, gate_chunk_elems=(N // chunks) * K)
    _release_later(b_src, b, flags, 2, side)
    fused_gemm(a, b, out, gate=gate)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert rel_err(out, a.float() @ b_src.float().t()) < 1e-2


@pytest.mark.parametrize("world,Tl,N,K", [(2, 512, 640, 512), (4, 256, 1024, 384), (8, 128, 512, 256)])
def test_scatter_epilogue_stores_rows_at_their_owner(world, Tl, N, K):
    torch.manual_seed(2)
    M = world * Tl
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    slots = [torch.full((Tl, N), float("nan"), device=DEV, dtype=torch.bfloat16) for _ in range(world)]
    dummy = torch.empty(1, dtype=torch.bfloat16, device=DEV).expand(M, N)
    fused_gemm(a, b, dummy, scatter=([s.data_ptr() for s in slots], Tl))
    torch.cuda.synchronize()
    ref = a.float() @ b.float().t()
    for r in range(world):
        assert rel_err(slots[r], ref[r * Tl:(r + 1) * Tl]) < 1e-2


@pytest.mark.parametrize("R,f32", [(1, True), (2, False), (4, True), (8, True), (8, False)])
@pytest.mark.parametrize("accumulate,store", [(False, True), (True, True), (False, False)])
def test_rs_adamw_matches_mean_and_torch_adamw(R, f32, accumulate, store):
    torch.manual_seed(3)
    C = native()
    n, shard_rank = 8192, 1 if R > 1 else 0
    dt = torch.float32 if f32 else torch.bfloat16
    bufs = [torch.randn(R * n, device=DEV).to(dt) for _ in range(R)]
    prev = torch.randn(n, device=DEV)
    grad = prev.clone()
    master = torch.randn(n, device=DEV)
    m = torch.randn(n, device=DEV) * 0.1
    v = torch.rand(n, device=DEV) * 0.1
    p16 = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    # three segments: decayed, not decayed, and an untouched tail (alignment padding)
    segs = torch.tensor([[0, 5000, 1e-3, 0.1], [5000, 8000, 1e-3, 0.0]], dtype=torch.float64)
    step = 3
    ref_m, ref_v, ref_p = m.clone(), v.clone(), master.clone()
    gs = grad if (accumulate or store) else grad[:0]   # no gradient shard at all
    C.rs_adamw([b.data_ptr() for b in bufs], shard_rank * n, n, f32, 1.0 / R, accumulate, gs,
               store, master, m, v, p16, segs, 0.9, 0.95, 1e-8, step)
    torch.cuda.synchronize()
    g = sum(b[shard_rank * n:(shard_rank + 1) * n].float() for b in bufs) / R
    if accumulate:
        g = g + prev
    if store:
        assert torch.allclose(grad, g, atol=1e-5, rtol=1e-5)
    else:
        assert torch.equal(grad, prev)
    # torch.optim.AdamW on the same state, one segment at a time
    for (s, e, lr, wd) in segs.tolist():
        s, e = int(s), int(e)
        p = torch.nn.Parameter(ref_p[s:e].clone())
        opt = torch.optim.AdamW([p], lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=wd)
        opt.state[p] = {"step": torch.tensor(float(step - 1)), "exp_avg": ref_m[s:e].clone(),
                        "exp_avg_sq": ref_v[s:e].clone()}
        p.grad = g[s:e].clone()
        opt.step()
        assert torch.allclose(master[s:e], p.detach(), atol=1e-6, rtol=1e-5)
        assert torch.allclose(m[s:e], opt.state[p]["exp_avg"], atol=1e-6, rtol=1e-5)
        assert torch.allclose(v[s:e], opt.state[p]["exp_avg_sq"], atol=1e-7, rtol=1e-5)
        assert torch.equal(p16[s:e], p.detach().to(torch.bfloat16))
    # outside every segment the state is untouched
    assert torch.equal(master[8000:], ref_p[8000:]) and torch.equal(m[8000:], ref_m[8000:])


def test_flag_wait_times_out_then_recovers():
    """The bounded wait of the tensor-parallel path: a peer that never publishes (a flag
    nothing sets) ends the wait after its limit with code base + peer index."""
    dev = torch.device(DEV, 0)
    C = native()
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    flags[0] = 7
    flags[1] = 9
    flags[3] = 7
    C.wait_flags_geq([flags.data_ptr() + 4 * i for i in range(4)], 7, error_flag(dev), 200, 200)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeoutError, match="code 202"):
        check_kernel_errors(dev)
    # the context is still usable; once the flag is set the same wait returns at once
    flags[2] = 8
    C.wait_flags_geq([flags.data_ptr() + 4 * i for i in range(4)], 7, error_flag(dev), 200, 200)
    x = torch.ones(1024, device=dev) * 2
    torch.cuda.synchronize()
    check_kernel_errors(dev)
    assert float(x.sum()) == 2048.0


def test_host_wait_is_bounded():
    """The ZeRO-3 run-ahead throttle waits for this GPU's own work with a deadline."""
    from femtotron_b200.sharding.zero3 import HostWaitTimeout, wait_event_bounded
    dev = torch.device(DEV, 0)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    native().wait_flags_geq([flag.data_ptr()], 1, error_flag(dev), 1000, 300)   # ~1 s, then gives up
    ev = torch.cuda.Event()
    ev.record()
    with pytest.raises(HostWaitTimeout):
        wait_event_bounded(ev, 0.1, "test")
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeoutError, match="code 300"):
        check_kernel_errors(dev)


def test_ag_pull_gathers_every_chunk_and_feeds_the_gated_gemm():
    """The tensor-parallel all-gather pull kernel with four emulated ranks: the peers' staged
    chunks (local tensors) land in ring order in the gathered buffer, each chunk counter
    reaches epoch x CTAs, and a GEMM gated on those counters, launched while the peers'
    READY flags are still unset, computes on the gathered rows."""
    C = native()
    dev = torch.device(DEV, 0)
    world, me, Tl, H, N, e = 4, 1, 512, 640, 768, 3
    ctas = int(C.gate_reserved_sms())
    torch.manual_seed(4)
    chunks = [torch.randn(Tl, H, device=dev).to(torch.bfloat16) for _ in range(world)]
    w = torch.randn(N, H, device=dev).to(torch.bfloat16)
    ready = torch.zeros(world, dtype=torch.int32, device=dev)
    # every epoch adds one count per CTA: after epochs 1..e-1 a counter holds (e-1) x CTAs
    count = torch.full((world,), (e - 1) * ctas, dtype=torch.int32, device=dev)
    full = torch.zeros(world * Tl, H, device=dev, dtype=torch.bfloat16)
    out = torch.empty(world * Tl, N, device=dev, dtype=torch.bfloat16)
    side, rel = torch.cuda.Stream(), torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    rel.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(rel):            # the peers publish about 10 ms later
        torch.cuda._sleep(20_000_000)
        for r in range(world):
            C.stream_write(ready.data_ptr() + 4 * r, e)
    with torch.cuda.stream(side):
        C.ag_pull([c.data_ptr() for c in chunks], [ready.data_ptr() + 4 * r for r in range(world)],
                  full, Tl * H * 2, count.data_ptr(), me, e, ctas, error_flag(dev), 5000)
    gate = dict(gate_flags=count.data_ptr(), gate_op=1, gate_epoch=e * ctas, gate_off=0,
                gate_row_elems=H, gate_chunk_elems=Tl * H, gate_rot_rows=me * Tl)
    fused_gemm(full, w, out, gate=gate)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.current_stream().wait_stream(rel)
    torch.cuda.synchronize()
    want = torch.cat(chunks)
    assert torch.equal(full, want)
    assert count.tolist() == [e * ctas] * world
    assert rel_err(out, want.float() @ w.float().t()) < 1e-2


def test_rs_pull_sums_every_rank_partial_of_its_rows():
    C = native()
    dev = torch.device(DEV, 0)
    world, me, Tl, N, e = 4, 2, 256, 1024, 5
    torch.manual_seed(5)
    parts = [torch.randn(world * Tl, N, device=dev).to(torch.bfloat16) for _ in range(world)]
    resid = torch.randn(Tl, N, device=dev).to(torch.bfloat16)
    flags = torch.full((world,), e, dtype=torch.int32, device=dev)
    out = torch.empty(Tl, N, device=dev, dtype=torch.bfloat16)
    off = me * Tl * N * 2
    C.rs_pull([p.data_ptr() + off for p in parts], [flags.data_ptr() + 4 * r for r in range(world)],
              resid.reshape(-1), out, Tl * N, e, error_flag(dev), 2000)
    torch.cuda.synchronize()
    want = sum(p[me * Tl:(me + 1) * Tl].float() for p in parts) + resid.float()
    assert rel_err(out, want) < 5e-3
    # a peer that never publishes: the reduction gives up with code 240 + peer
    flags[3] = e - 1
    C.rs_pull([p.data_ptr() + off for p in parts], [flags.data_ptr() + 4 * r for r in range(world)],
              None, out, Tl * N, e, error_flag(dev), 200)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeoutError, match="code 243"):
        check_kernel_errors(dev)


@pytest.mark.parametrize("M,N,K", [(1024, 768, 512), (2048, 4096, 1024), (1536, 256, 384), (4096, 1920, 640)])
@pytest.mark.parametrize("rot", [256, 512, 768])
def test_tile_order_rotation_keeps_the_product(M, N, K, rot):
    """Starting the tile order at another row block (as the all-gather GEMM does, at its own
    chunk) changes only the order in which tiles are computed."""
    torch.manual_seed(6)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    fused_gemm(a, b, out, gate=dict(gate_rot_rows=rot))
    torch.cuda.synchronize()
    assert rel_err(out, a.float() @ b.float().t()) < 1e-2
