# The allocation-free fused linear cross-entropy entry point, called through
# its exported C symbols the way a caller that cannot allocate would -- for
# example a host runtime whose own allocator owns the device's memory, or a
# latency-critical loop that must stay out of the driver's allocation paths:
# every buffer is supplied by the caller and the routine's own working memory
# is a fixed device array inside the library.  Checked against the regular
# fused_linear_ce op on two calls in a row (the second call must not see
# stale accumulators from the first), on one chunk of rows and on several
# (the chunk loop: dW accumulated across chunks, row offsets, the per-row
# buffers reused), with the device's free memory unchanged across a call and
# the device status word clean.  The file name sorts last so a run that stops
# at the first failure has already run every other test.
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from vagus_b200.ops import build, native
    native()                                   # loads (or builds) the extension
    lib = ctypes.CDLL(str(build.BUILD_DIR / f"{build.NAME}.so"))
    fn = lib.vagus_fused_linear_ce_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.vagus_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    status = lib.vagus_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return fn, err, status


def _device_status(status_fn, stream) -> int:
    word = ctypes.c_int(-1)
    rc = status_fn(stream, ctypes.byref(word))
    assert rc == 0, rc
    return word.value


@pytest.mark.parametrize("N,D,V", [(1000, 256, 4096), (1500, 256, 32768)])
def test_noalloc_ce_matches_fused_op_twice(N, D, V):
    from vagus_b200 import ops
    fn, err, status_fn = _lib()
    torch.manual_seed(0)
    z = 1e-3
    h = torch.randn(N, D, device="cuda").bfloat16()
    w32 = 0.05 * torch.randn(V, D, device="cuda")
    t = torch.randint(0, V, (N,), device="cuda")
    t[7] = -1                                   # an ignored row
    # regular entry point (allocates its own logits chunk)
    hr = h.clone().requires_grad_(True)
    wr = w32.clone().requires_grad_(True)
    loss_ref, z_ref = ops.fused_linear_ce(hr, wr, t, z_loss=z)
    loss_ref.backward()
    w16 = w32.bfloat16().contiguous()
    stream = torch.cuda.current_stream().cuda_stream
    loss = torch.zeros(2, device="cuda")
    dh = torch.empty(N, D, device="cuda", dtype=torch.bfloat16)
    dW = torch.zeros(V, D, device="cuda")
    for call in range(2):
        dW.zero_()
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = fn(h.data_ptr(), w16.data_ptr(), t.data_ptr(), N, D, V, z, loss.data_ptr(), dh.data_ptr(),
                dW.data_ptr(), stream)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        if call == 1:                           # after the first call's one-time set-up
            assert torch.cuda.mem_get_info()[0] == free0, "the call allocated device memory"
        assert _device_status(status_fn, stream) == 0
        assert abs(loss[0].item() - loss_ref.item()) < 2e-3 * max(1.0, abs(loss_ref.item()))
        assert abs(loss[1].item() - z_ref.item()) < 1e-3
        rel_h = ((dh.float() - hr.grad.float()).norm() / hr.grad.float().norm()).item()
        rel_w = ((dW - wr.grad).norm() / wr.grad.norm()).item()
        assert rel_h < 3e-2 and rel_w < 3e-2, (rel_h, rel_w)
        assert dh[7].abs().max().item() == 0.0  # the ignored row has no gradient


def test_noalloc_ce_reports_out_of_range_target():
    fn, err, status_fn = _lib()
    N, D, V = 256, 64, 1024
    h = torch.randn(N, D, device="cuda").bfloat16()
    w = torch.randn(V, D, device="cuda").bfloat16()
    t = torch.randint(0, V, (N,), device="cuda")
    t[3] = V + 5
    loss = torch.zeros(2, device="cuda")
    dh = torch.empty(N, D, device="cuda", dtype=torch.bfloat16)
    dW = torch.zeros(V, D, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(h.data_ptr(), w.data_ptr(), t.data_ptr(), N, D, V, 0.0, loss.data_ptr(), dh.data_ptr(), dW.data_ptr(),
            stream)
    assert rc == 0, err(rc).decode()
    assert _device_status(status_fn, stream) == 16            # the bad row was ignored and reported
    assert dh[3].abs().max().item() == 0.0 and torch.isfinite(loss).all()
    t[3] = 0                                                  # the next call starts with a clean status
    rc = fn(h.data_ptr(), w.data_ptr(), t.data_ptr(), N, D, V, 0.0, loss.data_ptr(), dh.data_ptr(), dW.data_ptr(),
            stream)
    assert rc == 0 and _device_status(status_fn, stream) == 0


def test_noalloc_ce_rejects_oversized_vocab_and_bad_splits():
    fn, err, _ = _lib()
    N, D, V = 256, 64, 1 << 20                # 128 rows x 2 MiB of logits exceed the scratch array
    rc = fn(1, 1, 1, N, D, V, 0.0, 1, 1, 1, None)   # rejected before any pointer is touched
    assert rc == -2 and b"too large" in err(rc)
    # V = 96 K: a chunk holds 128 rows, so N = 200 cannot split into chunks of >= 128 rows
    rc = fn(1, 1, 1, 200, 64, 96 * 1024, 0.0, 1, 1, 1, None)
    assert rc == -5 and b"256" in err(rc)
