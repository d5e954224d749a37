"""The allocation-free C entry point ``ft_xent_mean_loss_noalloc`` (for callers that cannot
allocate GPU memory themselves; see femtotron_b200/csrc/xent_noalloc.h) called through its
exported C symbol, checked against the regular cross-entropy path of the library
(xent_stats kernel + the loss reduction used by the LM-head function) on two calls in a
row.  The file is named to be collected last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import femtotron_b200._C as ext  # the extension that exports the symbol
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.ft_xent_mean_loss_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _existing_loss(logits, labels):
    from femtotron_b200.ops import kernels as K
    st = K.xent_stats(logits, labels, 0)
    lse = st[:, 0] + torch.log(st[:, 1])
    valid = labels != -100
    return torch.where(valid, lse - st[:, 2], torch.zeros_like(lse)).sum() / valid.sum()


def test_noalloc_loss_matches_existing_entry_point_twice():
    fn = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    for call, (T, V) in enumerate([(1000, 4096), (517, 32000)]):
        g = torch.Generator(device="cpu").manual_seed(100 + call)
        logits = (3 * torch.randn(T, V, generator=g)).to(torch.bfloat16).to(dev)
        labels = torch.randint(0, V, (T,), generator=g).to(dev)
        labels[::5] = -100
        out = torch.full((1,), float("nan"), device=dev)
        rc = fn(logits.data_ptr(), labels.data_ptr(), T, V, logits.stride(0), -100,
                out.data_ptr(), stream.cuda_stream)
        assert rc == 0, f"call {call}: return code {rc}"
        ref = _existing_loss(logits, labels)
        torch.cuda.synchronize()
        assert abs(out.item() - ref.item()) <= 1e-4 * abs(ref.item()), (call, out.item(), ref.item())


def test_noalloc_rejects_rows_beyond_maximum():
    fn = _lib()
    dev = torch.device("cuda", 0)
    logits = torch.zeros(8, 8, dtype=torch.bfloat16, device=dev)
    labels = torch.zeros(8, dtype=torch.long, device=dev)
    out = torch.zeros(1, device=dev)
    rc = fn(logits.data_ptr(), labels.data_ptr(), 65537, 8, 8, -100, out.data_ptr(), None)
    assert rc == 1
