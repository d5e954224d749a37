"""Kernel micro-benchmark and roofline report for the native sm_100a kernels.

    python -m femtotron_b200.utils.kbench all            # every op, Llama-3-8B shapes
    python -m femtotron_b200.utils.kbench gemm_qkv --iters 20
    python -m femtotron_b200.utils.kbench flash_fwd flash_fwd_v1 adamw   # several ops
    python -m femtotron_b200.utils.kbench flash_fwd --compare   # also time the torch library op

Each op is timed with CUDA events on the launching stream after warm-up, with a synchronize
on both sides; inputs are larger than L2 (126 MB) where the op is memory-bound, otherwise an
L2-sized buffer is rewritten between iterations.  The report gives achieved TFLOP/s or GB/s and
the fraction of the measured peaks (MEASURED_PEAKS.json at the repository root when present,
else the pool's fallback of 6.65 TB/s and 1.59 PFLOP/s).  One JSON line per op.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.nn.functional as F

from femtotron_b200.ops import kernels as K
from femtotron_b200.ops.ext import check_kernel_errors, error_flag, native
from femtotron_b200.ops.matmul import gemm

# Llama-3-8B, one micro-batch of 4096 tokens
T, H, FF, V, NQ, NKV, D = 4096, 4096, 14336, 128256, 32, 8, 128


def peaks() -> dict:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"tflops": float(d["bf16_tflops"]), "gbs": float(d["hbm_gbs"]), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1590.0, "gbs": 6650.0, "src": "fallback"}


_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def timed(fn, iters: int, warmup: int = 3, flush: bool = False) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if flush:
            flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def bf(*shape):
    return torch.randn(*shape, device="cuda", dtype=torch.bfloat16)


def op_gemm(name, M, N, K_, a_mn=False, b_mn=False, mode="store_bf16"):
    a = bf(K_, M) if a_mn else bf(M, K_)
    b = bf(K_, N) if b_mn else bf(N, K_)
    out = torch.empty(M, N, device="cuda",
                      dtype=torch.float32 if mode.endswith("f32") else torch.bfloat16)

    def run():
        gemm(a, b, out, a_mn=a_mn, b_mn=b_mn, mode=mode)

    def lib():
        aa = a.t() if a_mn else a
        bb = b if b_mn else b.t()
        torch.mm(aa, bb)
    return {"kind": "flops", "flops": 2.0 * M * N * K_, "run": run, "lib": lib, "name": name}


def op_flash(name, bwd: bool, variant: int = 0):
    B, S = 1, T
    qkv = bf(B * S, (NQ + 2 * NKV) * D)
    o = torch.empty(B * S, NQ * D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, NQ, S, device="cuda", dtype=torch.float32)
    err = error_flag(qkv.device)
    fl = 4.0 * B * NQ * S * S * D / 2
    q = qkv[:, : NQ * D].view(B, S, NQ, D).transpose(1, 2)
    k = qkv[:, NQ * D:(NQ + NKV) * D].view(B, S, NKV, D).transpose(1, 2)
    v = qkv[:, (NQ + NKV) * D:].view(B, S, NKV, D).transpose(1, 2)
    if not bwd:
        def run():
            native().flash_fwd_variant(qkv, o, lse, B, S, NQ, NKV, D, err, variant)

        def lib():
            F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        return {"kind": "flops", "flops": fl, "run": run, "lib": lib, "name": name}
    native().flash_fwd(qkv, o, lse, B, S, NQ, NKV, D, err)
    do = bf(B * S, NQ * D)
    dqkv = torch.empty_like(qkv)
    qq, kk, vv = [x.detach().clone().requires_grad_(True) for x in (q, k, v)]
    out = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=True)
    go = torch.randn_like(out)

    def run():
        native().flash_bwd(qkv, o, do, lse, dqkv, B, S, NQ, NKV, D, err)

    def lib():
        torch.autograd.grad(out, (qq, kk, vv), go, retain_graph=True)
    return {"kind": "flops", "flops": 2.5 * fl, "run": run, "lib": lib, "name": name}


def op_rmsnorm(name, bwd: bool):
    x, w = bf(4 * T, H), torch.ones(H, device="cuda", dtype=torch.bfloat16)
    if not bwd:
        def run():
            K.rmsnorm_fwd(x, w, 1e-5)
        return {"kind": "bytes", "bytes": 2.0 * x.numel() * 2 + 4 * x.shape[0], "run": run, "name": name}
    y, rstd = K.rmsnorm_fwd(x, w, 1e-5)
    dy = bf(4 * T, H)

    def run():
        K.rmsnorm_bwd(dy, x, w, rstd)
    return {"kind": "bytes", "bytes": 3.0 * x.numel() * 2, "run": run, "name": name}


def op_swiglu(name):
    gu = bf(4 * T, 2 * FF)

    def run():
        K.swiglu_fwd(gu, FF)
    return {"kind": "bytes", "bytes": gu.numel() * 2 * 1.5, "run": run, "name": name}


def op_adamw(name):
    n = 218 * 1000 * 1000  # one Llama-3-8B decoder layer
    p, m, v, g = (torch.randn(n, device="cuda") for _ in range(4))
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)

    def run():
        K.adamw_multi([p], [m], [v], [g], [out], [0.1], lr=1e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                      step=10)
    # read p, m, v, g (fp32), write p, m, v (fp32) + bf16 copy
    return {"kind": "bytes", "bytes": n * (4 * 4 + 3 * 4 + 2), "run": run, "name": name}


def op_xent(name):
    logits = bf(T, V)
    labels = torch.randint(0, V, (T,), device="cuda")

    def run():
        K.xent_stats(logits, labels, 0)
    return {"kind": "bytes", "bytes": logits.numel() * 2, "run": run, "name": name}


def op_p2p_copy(name, streams: int):
    """Copy-engine peer copy cuda:1 -> cuda:0 of one ZeRO-3 unit half (218 MB), split over
    `streams` streams (needs two visible GPUs)."""
    n = 109 * 1000 * 1000
    src = torch.randn(n, device="cuda:1").to(torch.bfloat16)
    dst = torch.empty(n, device="cuda:0", dtype=torch.bfloat16)
    ss = [torch.cuda.Stream(device="cuda:0") for _ in range(streams)]
    parts = list(zip(dst.chunk(streams), src.chunk(streams)))

    def run():
        cur = torch.cuda.current_stream()
        for st, (d, s_) in zip(ss, parts):
            st.wait_stream(cur)
            with torch.cuda.stream(st):
                d.copy_(s_, non_blocking=True)
        for st in ss:
            cur.wait_stream(st)
    return {"kind": "bytes", "bytes": n * 2, "run": run, "name": name}


# ---- fused communication kernels, emulated on one GPU: every "peer" buffer is a local one
# and every flag is already published, so the kernels run their full code path (flag checks,
# per-owner addressing) against local HBM instead of NVLink.  Shapes: Llama-2-13B with TP=8 and
# sequence parallelism (micro-batch 2, seq 4096) and one Llama-3-8B ZeRO-3 unit at DP=8.
TP, T13, H13, QKV13 = 8, 2 * 4096, 5120, 3 * 5120 // 8


def op_gemm_gated(name):
    """All-gather -> GEMM: the QKV projection whose A rows (the sequence-parallel activations)
    arrive in TP chunks; the producer checks chunk flags before each A tile."""
    from femtotron_b200.parallel.tensor_parallel.fused import fused_gemm
    a, b = bf(T13, H13), bf(QKV13, H13)
    out = torch.empty(T13, QKV13, device="cuda", dtype=torch.bfloat16)
    flags = torch.ones(TP, dtype=torch.int32, device="cuda")
    gate = dict(gate_flags=flags.data_ptr(), gate_op=1, gate_epoch=1, gate_off=0,
                gate_row_elems=H13, gate_chunk_elems=(T13 // TP) * H13)

    def run():
        fused_gemm(a, b, out, gate=gate)
    # `keep` holds the flag tensor alive: the kernel only receives its address
    return {"kind": "flops", "flops": 2.0 * T13 * QKV13 * H13, "run": run, "name": name, "keep": flags}


def op_gemm_scatter(name):
    """GEMM -> reduce-scatter: the o_proj partial product whose rows are stored straight into
    their owner rank's slot (here TP local slots)."""
    from femtotron_b200.parallel.tensor_parallel.fused import fused_gemm
    k = H13 // TP
    a, b = bf(T13, k), bf(H13, k)
    out = torch.empty(T13, H13, device="cuda", dtype=torch.bfloat16)
    slots = torch.empty(TP, T13 // TP, H13, device="cuda", dtype=torch.bfloat16)
    ptrs = [slots[r].data_ptr() for r in range(TP)]

    def run():
        fused_gemm(a, b, out, scatter=(ptrs, T13 // TP))
    return {"kind": "flops", "flops": 2.0 * T13 * H13 * k, "run": run, "name": name, "keep": slots}


def op_rs_p2p(name):
    """ZeRO-3 gradient reduce-scatter with the fp32 cast, 1/dp scale and the AdamW update of
    the shard fused (``rs_adamw``): one Llama-3-8B unit (218 M parameters, fp32 gradients) at
    DP=8, this rank's slice.  The eight sources are local buffers here (one GPU)."""
    R, shard = 8, 218 * 1000 * 1000 // 8 // 8 * 8
    # rank 0 reads elements [0, shard) of every peer's buffer: allocate only that slice
    bufs = [torch.randn(shard, device="cuda") for _ in range(R)]
    grad = torch.zeros(shard, device="cuda")
    master = torch.randn(shard, device="cuda")
    m, v = torch.zeros_like(master), torch.zeros_like(master)
    p16 = torch.empty(shard, device="cuda", dtype=torch.bfloat16)
    segs = torch.tensor([[0, shard, 1e-4, 0.01]], dtype=torch.float64)
    ptrs = [b.data_ptr() for b in bufs]

    def run():
        native().rs_adamw(ptrs, 0, shard, True, 1.0 / R, False, grad, True, master, m, v, p16,
                          segs, 0.9, 0.95, 1e-8, 1)
    run.keep = bufs   # the peer buffers are passed by address only
    # read R slices + master/m/v, write grad/master/m/v (fp32) and the bf16 shard
    return {"kind": "bytes", "bytes": shard * (4 * R + 12 + 16 + 2), "run": run, "name": name}


def op_tp_ag_pull(name, world=8):
    """The tensor-parallel all-gather pull kernel alone (``ag_pull``) with every "peer" chunk
    in local memory: Llama-2-13B, TP=8 + SP, 1024 tokens x 5120 per rank; READY flags preset."""
    C = native()
    from femtotron_b200.ops.ext import error_flag
    Tl, H = 1024, 5120
    chunks = [torch.randn(Tl, H, device="cuda").to(torch.bfloat16) for _ in range(world)]
    full = torch.empty(world * Tl, H, device="cuda", dtype=torch.bfloat16)
    ready = torch.ones(world, dtype=torch.int32, device="cuda")
    count = torch.zeros(world, dtype=torch.int32, device="cuda")
    ctas = int(C.gate_reserved_sms())
    ptrs = [c.data_ptr() for c in chunks]

    def run():
        C.ag_pull(ptrs, [ready.data_ptr() + 4 * r for r in range(world)], full, Tl * H * 2,
                  count.data_ptr(), 0, 1, ctas, error_flag(full.device), 1000)
    run.keep = chunks
    return {"kind": "bytes", "bytes": 2 * world * Tl * H * 2, "run": run, "name": name}


def op_tp_rs_pull(name, world=8):
    """The tensor-parallel reduce-scatter pull (``rs_pull``) with every rank's partial in
    local memory: this rank's 1024 rows x 5120 of eight partials, plus the residual."""
    C = native()
    from femtotron_b200.ops.ext import error_flag
    Tl, N = 1024, 5120
    parts = [torch.randn(Tl, N, device="cuda").to(torch.bfloat16) for _ in range(world)]
    resid = torch.randn(Tl, N, device="cuda").to(torch.bfloat16)
    out = torch.empty(Tl, N, device="cuda", dtype=torch.bfloat16)
    flags = torch.ones(world, dtype=torch.int32, device="cuda")
    ptrs = [p.data_ptr() for p in parts]

    def run():
        C.rs_pull(ptrs, [flags.data_ptr() + 4 * r for r in range(world)], resid.reshape(-1), out,
                  Tl * N, 1, error_flag(out.device), 1000)
    run.keep = parts
    return {"kind": "bytes", "bytes": (world + 2) * Tl * N * 2, "run": run, "name": name}


OPS = {
    "p2p_copy_1": lambda: op_p2p_copy("p2p_copy_1", 1),
    "p2p_copy_4": lambda: op_p2p_copy("p2p_copy_4", 4),
    "gemm_qkv": lambda: op_gemm("gemm_qkv", T, (NQ + 2 * NKV) * D, H),
    "gemm_o": lambda: op_gemm("gemm_o", T, H, NQ * D),
    "gemm_gateup": lambda: op_gemm("gemm_gateup", T, 2 * FF, H),
    "gemm_down": lambda: op_gemm("gemm_down", T, H, FF),
    "gemm_lmhead": lambda: op_gemm("gemm_lmhead", T, V, H),
    "gemm_dgrad_gateup": lambda: op_gemm("gemm_dgrad_gateup", T, H, 2 * FF, b_mn=True),
    "gemm_wgrad_gateup": lambda: op_gemm("gemm_wgrad_gateup", 2 * FF, H, T, a_mn=True, b_mn=True,
                                         mode="acc_f32"),
    "flash_fwd": lambda: op_flash("flash_fwd", False),
    # forward variants: one query tile per CTA; two tiles reading S once (the default reads it
    # twice); two tiles with a quarter of the exponentials on the FMA pipe
    "flash_fwd_v1": lambda: op_flash("flash_fwd_v1", False, 1),
    "flash_fwd_1pass": lambda: op_flash("flash_fwd_1pass", False, 3),
    "flash_fwd_emu": lambda: op_flash("flash_fwd_emu", False, 4),
    "flash_bwd": lambda: op_flash("flash_bwd", True),
    "rmsnorm_fwd": lambda: op_rmsnorm("rmsnorm_fwd", False),
    "rmsnorm_bwd": lambda: op_rmsnorm("rmsnorm_bwd", True),
    "swiglu_fwd": lambda: op_swiglu("swiglu_fwd"),
    "adamw": lambda: op_adamw("adamw"),
    "gemm_gated_ag": lambda: op_gemm_gated("gemm_gated_ag"),
    "gemm_scatter_rs": lambda: op_gemm_scatter("gemm_scatter_rs"),
    "rs_p2p": lambda: op_rs_p2p("rs_p2p"),
    "tp_ag_pull": lambda: op_tp_ag_pull("tp_ag_pull"),
    "tp_rs_pull": lambda: op_tp_rs_pull("tp_rs_pull"),
    "xent_stats": lambda: op_xent("xent_stats"),
}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("op", nargs="+", choices=sorted(OPS) + ["all"])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--compare", action="store_true", help="also time the torch library op")
    args = ap.parse_args(argv)
    pk = peaks()
    names = (sorted(n for n in OPS if not n.startswith("p2p")) if "all" in args.op
             else list(dict.fromkeys(args.op)))
    for n in names:
        spec = OPS[n]()
        flush = spec["kind"] == "flops"  # memory-bound ops already use inputs larger than L2
        ms = timed(spec["run"], args.iters, args.warmup, flush=flush)
        check_kernel_errors()
        rec = {"op": n, "ms": round(ms, 4)}
        if spec["kind"] == "flops":
            tf = spec["flops"] / ms / 1e9
            rec.update(tflops=round(tf, 1), frac_of_peak=round(tf / pk["tflops"], 3))
            if args.compare and "lib" in spec:
                lms = timed(spec["lib"], args.iters, args.warmup, flush=True)
                rec.update(lib_ms=round(lms, 4), lib_tflops=round(spec["flops"] / lms / 1e9, 1))
        else:
            gbs = spec["bytes"] / ms / 1e6
            rec.update(gbs=round(gbs, 1), frac_of_peak=round(gbs / pk["gbs"], 3))
        rec["peak_src"] = pk["src"]
        print(json.dumps(rec), flush=True)
        del spec
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
