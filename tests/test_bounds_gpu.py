"""The bounds-checked build (VAGUS_BOUNDS_CHECK=1; see ops/build.py): an
index outside its tensor is recorded in the device error word as kErrBounds
(32) and the access is skipped -- so a bad token id reports instead of
reading past the embedding table.  Skipped in the normal build, where the
checks compile to nothing; the GPU suite is run once under this build."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_out_of_range_token_is_reported_and_skipped():
    from vagus_b200 import ops
    C = ops.native()
    if not C.bounds_checked():
        pytest.skip("normal build: bounds checks are compiled out (run with VAGUS_BOUNDS_CHECK=1)")
    V, D = 64, 128
    W = torch.randn(V, D, device="cuda")
    tok = torch.tensor([3, V + 7, 5], device="cuda")
    torch.cuda.synchronize()
    C.reset_error()
    y = C.embedding_fwd(W, tok, True)
    torch.cuda.synchronize()
    assert C.error_word() == 32
    C.reset_error()
    assert torch.equal(y[0], W[3]) and torch.equal(y[2], W[5])
    dW = torch.zeros(V, D, device="cuda")
    C.embedding_bwd(torch.ones(3, D, device="cuda"), tok, dW)
    torch.cuda.synchronize()
    assert C.error_word() == 32 and dW.sum().item() == 2 * D      # the bad row added nothing
    C.reset_error()
