"""The allocation-free C entry point ``ft_xent_mean_loss_noalloc``, for callers that cannot
allocate GPU memory themselves (a C or foreign-language host runtime without PyTorch's
allocator, a process whose device memory another allocator reserved up front, a call site
where allocating is not allowed).  Its per-row scratch lives in a fixed device array of the
library; see femtotron_b200/csrc/xent_noalloc.h.

It is called here through its exported C symbol and checked against plain PyTorch:
``F.cross_entropy`` in fp32 on the same (bf16-valued) logits, on two calls in a row with
different shapes (the shared scratch keeps the previous call's rows), on a column-sliced
logits view (row stride larger than the vocabulary), and on the documented edge cases: no
valid row and zero rows give NaN, an out-of-range label gives NaN, and bad arguments are
refused without a launch.  The file is named to be collected last."""
import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    import femtotron_b200._C as ext  # the extension that exports the symbol
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.ft_xent_mean_loss_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _call(fn, logits, labels, vocab, out, stream):
    return fn(logits.data_ptr(), labels.data_ptr(), labels.numel(), vocab, logits.stride(0),
              -100, out.data_ptr(), stream.cuda_stream)


def _oracle(logits, labels):
    return F.cross_entropy(logits.float(), labels, ignore_index=-100)


def test_noalloc_loss_matches_fp32_cross_entropy_twice():
    fn = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    for call, (T, V) in enumerate([(1000, 4096), (517, 32000)]):
        g = torch.Generator(device="cpu").manual_seed(100 + call)
        logits = (3 * torch.randn(T, V, generator=g)).to(torch.bfloat16).to(dev)
        labels = torch.randint(0, V, (T,), generator=g).to(dev)
        labels[::5] = -100
        out = torch.full((1,), float("nan"), device=dev)
        rc = _call(fn, logits, labels, V, out, stream)
        assert rc == 0, f"call {call}: return code {rc}"
        ref = _oracle(logits, labels)
        torch.cuda.synchronize()
        assert abs(out.item() - ref.item()) <= 1e-4 * abs(ref.item()), (call, out.item(), ref.item())


def test_noalloc_strided_rows():
    """A column slice of a wider logits buffer: the row stride (ld) exceeds the vocabulary."""
    fn = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device="cpu").manual_seed(7)
    wide = (2 * torch.randn(300, 2048 + 64, generator=g)).to(torch.bfloat16).to(dev)
    logits = wide[:, :2048]
    labels = torch.randint(0, 2048, (300,), generator=g).to(dev)
    out = torch.full((1,), float("nan"), device=dev)
    assert _call(fn, logits, labels, 2048, out, stream) == 0
    ref = _oracle(logits, labels)
    torch.cuda.synchronize()
    assert abs(out.item() - ref.item()) <= 1e-4 * abs(ref.item())


def test_noalloc_edge_cases_give_nan():
    fn = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    logits = torch.randn(64, 512, device=dev).to(torch.bfloat16)
    out = torch.zeros(1, device=dev)
    # every row ignored: a mean over no rows
    ignored = torch.full((64,), -100, dtype=torch.long, device=dev)
    assert _call(fn, logits, ignored, 512, out, stream) == 0
    torch.cuda.synchronize()
    assert math.isnan(out.item())
    # zero rows
    out.zero_()
    empty = torch.empty(0, dtype=torch.long, device=dev)
    assert fn(logits.data_ptr(), empty.data_ptr(), 0, 512, 512, -100, out.data_ptr(),
              stream.cuda_stream) == 0
    torch.cuda.synchronize()
    assert math.isnan(out.item())
    # a label outside [0, vocab) that is not the ignore index
    out.zero_()
    bad = torch.randint(0, 512, (64,), device=dev)
    bad[10] = 512
    assert _call(fn, logits, bad, 512, out, stream) == 0
    torch.cuda.synchronize()
    assert math.isnan(out.item())
    # and a valid call afterwards is unaffected by the previous contents of the scratch
    good = torch.randint(0, 512, (64,), device=dev)
    assert _call(fn, logits, good, 512, out, stream) == 0
    ref = _oracle(logits, good)
    torch.cuda.synchronize()
    assert abs(out.item() - ref.item()) <= 1e-4 * abs(ref.item())


def test_noalloc_rejects_bad_arguments():
    fn = _lib()
    dev = torch.device("cuda", 0)
    logits = torch.zeros(16, 16, dtype=torch.bfloat16, device=dev)
    labels = torch.zeros(16, dtype=torch.long, device=dev)
    out = torch.full((1,), 5.0, device=dev)
    # more rows than the scratch array holds: refused before any launch
    assert fn(logits.data_ptr(), labels.data_ptr(), 65537, 16, 16, -100, out.data_ptr(), None) == 1
    # vocabulary not a multiple of 8
    assert fn(logits.data_ptr(), labels.data_ptr(), 16, 12, 16, -100, out.data_ptr(), None) == 2
    # logits pointer not 16-byte aligned
    assert fn(logits.data_ptr() + 2, labels.data_ptr(), 8, 8, 16, -100, out.data_ptr(), None) == 2
    # row stride smaller than the vocabulary
    assert fn(logits.data_ptr(), labels.data_ptr(), 8, 16, 8, -100, out.data_ptr(), None) == 2
    torch.cuda.synchronize()
    assert out.item() == 5.0   # nothing was written
