"""Timing of the fused tensor-parallel collectives against their roofline and against NCCL.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m femtotron_b200.utils.tp_bench \
        [--tokens 8192] [--hidden 5120] [--ffn 13824] [--heads 40] [--iters 20] [--json out.json]

For each sequence-parallel projection of one Llama-2-13B decoder layer at TP = world size
(tokens = micro-batch 2 x seq 4096 by default) it times, with CUDA events on the compute
stream and the maximum over ranks:

  * ``qkv_ag_gemm``     all-gather of the token-sharded input fused into the QKV GEMM
  * ``gateup_ag_gemm``  the same into the gate/up GEMM with the SwiGLU epilogue
  * ``o_gemm_rs``       o_proj GEMM whose epilogue scatters rows to their owners + owner sum
  * ``down_gemm_rs``    the same for down_proj

and the same math as NCCL ``all_gather_into_tensor`` + GEMM / GEMM + ``reduce_scatter_tensor``
(both arms use this library's GEMM).  Roofline of a fused op = the slower of its FLOPs at the
measured bf16 peak and the bytes that must cross NVLink at the measured 770 GB/s per direction
per GPU: (tp-1)/tp of the gathered (or scattered) activation.
"""
from __future__ import annotations

import argparse
import json
import os

import femtotron_b200  # noqa: F401
import torch
import torch.distributed as dist

NVLINK_GBS = 770.0   # measured peer copy per direction per GPU on this pool's B200s


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--ffn", type=int, default=13824)
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()

    from femtotron_b200.ops.ext import check_kernel_errors
    from femtotron_b200.ops.matmul import gemm
    from femtotron_b200.parallel.tensor_parallel.fused import SPColumnFn, SPRowFn, tp_fused_comm
    from femtotron_b200.utils.dist import init_distributed, max_over_ranks

    rank, world, local = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    T, H, F, nh = args.tokens, args.hidden, args.ffn, args.heads
    Tl = T // world
    d = H // nh
    qkv_n = 3 * (nh // world) * d
    Fl = F // world
    try:
        peak = json.load(open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")))["bf16_tflops"]
    except OSError:
        peak = 1590.0
    g = torch.Generator(device="cpu").manual_seed(rank)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16).to(dev)

    x_local = rnd(Tl, H)
    wq, wk, wv = rnd(qkv_n // 3, H), rnd(qkv_n // 3, H), rnd(qkv_n // 3, H)
    wg, wu = rnd(Fl, H), rnd(Fl, H)
    wo = rnd(H, qkv_n // 3)
    wd = rnd(H, Fl)
    h_attn = rnd(T, qkv_n // 3)
    h_mlp = rnd(T, Fl)
    comm = tp_fused_comm(dist.group.WORLD, Tl, max(H, H), dev)
    group = dist.group.WORLD

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b) / args.iters)

    ag_bytes = (world - 1) / world * T * H * 2
    results = {}

    def report(name, ms, flops, nbytes):
        roof = max(flops / (peak * 1e12), nbytes / (NVLINK_GBS * 1e9)) * 1e3
        results[name] = {"ms": round(ms, 4), "roofline_ms": round(roof, 4),
                         "fraction_of_roofline": round(roof / ms, 3),
                         "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                         "nvlink_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}

    with torch.no_grad():
        # fused paths (forward of the autograd functions)
        report("qkv_ag_gemm", timed(lambda: SPColumnFn.forward(_Ctx(), x_local, comm, "linear", None, wq, wk, wv)),
               2.0 * T * qkv_n * H, ag_bytes)
        report("gateup_ag_gemm", timed(lambda: SPColumnFn.forward(_Ctx(), x_local, comm, "swiglu", None, wg, wu)),
               2.0 * T * 2 * Fl * H, ag_bytes)
        report("o_gemm_rs", timed(lambda: SPRowFn.forward(_Ctx(), h_attn, None, comm, wo)),
               2.0 * T * H * (qkv_n // 3), ag_bytes)
        report("down_gemm_rs", timed(lambda: SPRowFn.forward(_Ctx(), h_mlp, None, comm, wd)),
               2.0 * T * H * Fl, ag_bytes)

        # NCCL baselines with the same GEMMs
        full = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        wqkv = torch.cat([wq, wk, wv])
        out_qkv = torch.empty(T, qkv_n, dtype=torch.bfloat16, device=dev)

        def nccl_qkv():
            dist.all_gather_into_tensor(full, x_local, group=group)
            gemm(full, wqkv, out_qkv)
        report("nccl_ag_then_qkv_gemm", timed(nccl_qkv), 2.0 * T * qkv_n * H, ag_bytes)
        part = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        red = torch.empty(Tl, H, dtype=torch.bfloat16, device=dev)

        def nccl_o():
            gemm(h_attn, wo, part)
            dist.reduce_scatter_tensor(red, part, group=group)
        report("nccl_o_gemm_then_rs", timed(nccl_o), 2.0 * T * H * (qkv_n // 3), ag_bytes)

        def nccl_down():
            gemm(h_mlp, wd, part)
            dist.reduce_scatter_tensor(red, part, group=group)
        report("nccl_down_gemm_then_rs", timed(nccl_down), 2.0 * T * H * Fl, ag_bytes)

    check_kernel_errors(dev)
    if rank == 0:
        out = {"world": world, "tokens": T, "hidden": H, "ffn": F, "heads": nh,
               "peak_tflops": peak, "nvlink_gbs": NVLINK_GBS, "ops": results}
        print(json.dumps(out), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(out, f, indent=1)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


class _Ctx:
    """Stand-in for an autograd context when the forward is called directly (no graph)."""

    def save_for_backward(self, *t):
        pass


if __name__ == "__main__":
    main()
