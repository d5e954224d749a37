"""2-GPU NVLS checks launched by tests/test_multigpu.py through torchrun: the in-switch
all-reduce (``parallel/nvls.py``) against NCCL's all-reduce on the same inputs (fp32 and bf16,
sum and mean, sizes that are not multiples of 16 bytes, repeated calls), the packed variant
used by the data-parallel buckets, and the bus bandwidth of both on 256 MB of bf16."""
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import femtotron_b200  # noqa: E402,F401
from femtotron_b200.ops.ext import check_kernel_errors  # noqa: E402
from femtotron_b200.parallel.nvls import NVLSAllReduce  # noqa: E402
from femtotron_b200.utils.dist import init_distributed, max_over_ranks  # noqa: E402


def main():
    rank, world, local = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    nv = NVLSAllReduce(dist.group.WORLD, 300 << 20, dev)
    res = {"world": world, "buffer_bytes": nv.data_bytes}
    worst = 0.0
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    for it in range(3):
        for dtype in (torch.float32, torch.bfloat16):
            for n in (8, 1000, 4099, 1 << 20):
                for avg in (False, True):
                    x = torch.randn(n, generator=g).to(dtype).to(dev)
                    ref = x.float().clone()
                    dist.all_reduce(ref)
                    if avg:
                        ref /= world
                    nv.all_reduce_(x, average=avg)
                    tol = 1e-5 if dtype == torch.float32 else 1e-2
                    err = ((x.float() - ref).abs().max() / (ref.abs().max() + 1e-6)).item()
                    worst = max(worst, err / tol)
    res["worst_err_over_tol"] = worst
    ts = [torch.randn(n, generator=g).to(dev) for n in (3, 1024, 77777)]
    refs = [t.clone() for t in ts]
    for r in refs:
        dist.all_reduce(r)
        r /= world
    nv.all_reduce_many_(ts, average=True)
    res["packed_ok"] = all(torch.allclose(a, b, atol=1e-6, rtol=1e-5) for a, b in zip(ts, refs))
    # bus bandwidth on 256 MB of bf16 (2 (n-1)/n x bytes / time, the NCCL convention)
    x = torch.randn(128 << 20, device=dev).to(torch.bfloat16)
    nbytes = x.numel() * 2

    def bw(fn, iters=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(a.elapsed_time(b) / iters)
        return ms, 2 * (world - 1) / world * nbytes / (ms * 1e-3) / 1e9
    res["nvls_ms"], res["nvls_busbw_gbs"] = bw(lambda: nv.all_reduce_(x))
    res["nccl_ms"], res["nccl_busbw_gbs"] = bw(lambda: dist.all_reduce(x))
    check_kernel_errors(dev)
    nv.close()
    if rank == 0:
        print("RESULT " + json.dumps(res), flush=True)
        out = os.environ.get("FT_TEST_RESULT_DIR")
        if out:
            with open(os.path.join(out, f"nvls_check_n{world}.json"), "w") as f:
                json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
