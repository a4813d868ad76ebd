"""q3_argmax_noalloc: the greedy argmax for callers that cannot let the
library allocate device memory (serving runtimes that plan every byte of
device memory themselves, hot loops that cannot take cudaMalloc's implicit
synchronisation).  Its scratch is a fixed array inside
the library; this checks it against q3_argmax, which allocates its own
scratch, through the C ABI, on two calls in a row -- the second call must
not be disturbed by what the first left in the shared array.

Kept in its own file, collected last, so a failure here never stops the
other tests from running first.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _argmax_both(logits_bits: np.ndarray):
    import torch

    from inference_b200._lib import check, lib

    L = lib()
    x = torch.from_numpy(logits_bits.view(np.int16)).cuda()
    idx_ref = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    idx_new = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    check(L.q3_argmax(x.data_ptr(), x.numel(), idx_ref.data_ptr(), s))
    check(L.q3_argmax_noalloc(x.data_ptr(), x.numel(), idx_new.data_ptr(), s))
    torch.cuda.synchronize()
    return int(idx_ref.item()), int(idx_new.item())


def _bf16(values: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def test_noalloc_argmax_matches_allocating_argmax_twice():
    rng = np.random.default_rng(2024)
    # call 1: a vocabulary-sized row whose maximum sits late, so every segment key matters
    a = _bf16(rng.uniform(-3, 3, 151936))
    a[150001] = 0x4120  # 10.0
    ref1, new1 = _argmax_both(a)
    assert new1 == ref1 == 150001
    # call 2: a shorter row with ties; keys left over from call 1 must not leak in
    b = _bf16(rng.uniform(-3, 1, 9000))
    b[[77, 4096, 8999]] = 0x4040  # 3.0 three times: the first index wins
    ref2, new2 = _argmax_both(b)
    assert new2 == ref2 == 77


def test_noalloc_argmax_size_limit():
    from inference_b200._lib import lib

    L = lib()
    # rejected on the host before any launch
    assert L.q3_argmax_noalloc(16, (1 << 24) + 1, 16, None) == 1
    assert b"16777216" in L.q3_last_error()
