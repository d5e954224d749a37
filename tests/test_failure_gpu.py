"""Bounded device-side waits (failure detection without a GPU fault): a kernel whose peer never
publishes its flag gives up after its time limit, records an error code that the host reads as
KernelTimeoutError, and leaves the CUDA context usable.  The 'peer' here is a flag word on the
same GPU that nothing sets; no second kernel is involved."""
import pytest
import torch

from femtotron_b200.ops.ext import KernelTimeoutError, check_kernel_errors, error_flag, native

pytestmark = pytest.mark.gpu


def test_reduce_scatter_flag_wait_times_out_then_recovers():
    dev = torch.device("cuda", 0)
    C = native()
    world, shard, rank, epoch = 2, 4096, 0, 1
    torch.manual_seed(0)
    bufs = [torch.randn(world * shard, device=dev).to(torch.bfloat16) for _ in range(world)]
    flags = torch.zeros(world, dtype=torch.int32, device=dev)   # this rank's flag array
    other = torch.zeros(world, dtype=torch.int32, device=dev)   # the absent peer's array
    flags[rank] = epoch                                          # own buffer published
    acc = torch.full((shard,), 7.0, device=dev)
    err = error_flag(dev)
    check_kernel_errors(dev)   # start clean

    ptrs = [b.data_ptr() for b in bufs]
    C.p2p_reduce_scatter(ptrs, flags.data_ptr(), [flags.data_ptr(), other.data_ptr()], acc, shard,
                         rank, epoch, 0.5, False, err, False, 200)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeoutError, match="code 101"):
        check_kernel_errors(dev)   # rank 1 never published
    assert torch.all(acc == 7.0)    # gave up before touching the output

    # the context is still usable: publish the peer's flag and run the same reduction
    flags[1] = epoch
    C.p2p_reduce_scatter(ptrs, flags.data_ptr(), [flags.data_ptr(), other.data_ptr()], acc, shard,
                         rank, epoch, 0.5, False, err, False, 200)
    torch.cuda.synchronize()
    check_kernel_errors(dev)
    want = 0.5 * (bufs[0][:shard].float() + bufs[1][:shard].float())
    assert torch.allclose(acc, want, atol=1e-6, rtol=1e-6)
