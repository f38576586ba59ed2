"""wsp_argmax_no_alloc against wsp_argmax: two calls in a row on different
inputs, each equal to the allocating entry point on the same inputs (and to
the masked argmax the oracle defines); later calls leave the device's free
memory unchanged; then the size limit of its fixed scratch.  Collected last, so it runs after every other test has used the
device, and it passes on its own too."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _device_argmax(entry, logits, mask):
    import torch
    rows, length = logits.shape
    dl = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    dm = torch.from_numpy(mask.astype(np.float32)).cuda() if mask is not None else None
    out = torch.full((rows,), 7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    entry(dl.data_ptr(), dm.data_ptr() if dm is not None else None, out.data_ptr(), rows, length)
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.uint32)


def _cases():
    rng = np.random.default_rng(5)
    wide = rng.standard_normal((40, 51864)).astype(np.float32)
    wide[3, [100, 40000]] = 9.0           # a tie: the lower index wins
    mask = np.zeros(51864, np.float32)
    mask[rng.choice(51864, 3000, replace=False)] = 1
    mask[100] = 0
    narrow = rng.standard_normal((7, 1000)).astype(np.float32)
    narrow[2] = -1.0                      # a constant row
    return [(wide, mask), (narrow, None)]


def test_two_calls_in_a_row_match_the_allocating_argmax():
    from whispereacp_b200 import argmax, argmax_no_alloc
    for logits, mask in _cases():
        static = _device_argmax(argmax_no_alloc, logits, mask)
        allocating = _device_argmax(argmax, logits, mask)
        assert np.array_equal(static, allocating)
        assert np.array_equal(static, O.masked_argmax(logits, mask))


def test_calls_after_the_first_take_no_device_memory():
    """The property the entry point exists for: once its first call on the
    device has looked its scratch up, later calls leave the device's free
    memory (cudaMemGetInfo) exactly where it was."""
    import torch
    from whispereacp_b200 import argmax_no_alloc
    logits, mask = _cases()[0]
    rows, length = logits.shape
    dl = torch.from_numpy(logits).cuda()
    dm = torch.from_numpy(mask).cuda()
    out = torch.empty((rows,), dtype=torch.int32, device="cuda")
    argmax_no_alloc(dl.data_ptr(), dm.data_ptr(), out.data_ptr(), rows, length)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(8):
        argmax_no_alloc(dl.data_ptr(), dm.data_ptr(), out.data_ptr(), rows, length)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert np.array_equal(out.cpu().numpy().astype(np.uint32), O.masked_argmax(logits, mask))


def test_more_rows_than_the_fixed_scratch_holds_are_refused():
    from whispereacp_b200 import argmax_no_alloc
    from whispereacp_b200._native import library
    groups = -(-51866 // 2048)
    rows = 65536 // groups + 1
    # Refused on the host before any pointer is used or anything launched.
    with pytest.raises(ValueError, match="at most 65536"):
        argmax_no_alloc(16, None, 16, rows, 51866)
    assert b"2521 rows of 51866" in library().wsp_last_error()
