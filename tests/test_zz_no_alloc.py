"""The allocation-free cross-entropy entry point (ns_cross_entropy_noalloc).

It serves callers that cannot call cudaMalloc when they run the loss, such as
code recording a CUDA graph or a host whose device memory belongs to another
allocator: its scratch is a static device array inside the library instead of
a caller workspace.  This file is named so that pytest collects it last; it
checks the entry point through the C ABI against ns_cross_entropy (which takes
a workspace) and against the oracle on two calls in a row, within the
tolerance the other tests use.  The rejection of sizes beyond the static
array needs no GPU and is checked in test_abi_errors.py.
"""

import numpy as np
import pytest
import torch

from neuralsuite_b200 import _lib
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import ATOL, RTOL, assert_close, normal, rng

pytestmark = pytest.mark.gpu


def noalloc(logits, targets, denom):
    lib = _lib.load()
    rows, classes = logits.shape
    loss = torch.empty(1, dtype=torch.float32, device=logits.device)
    d = torch.empty_like(logits)
    err = torch.zeros(1, dtype=torch.int32, device=logits.device)
    _lib.check(lib.ns_cross_entropy_noalloc(logits.data_ptr(), targets.data_ptr(), rows, classes,
                                            float(denom), loss.data_ptr(), d.data_ptr(),
                                            err.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
    return loss, d, err


def test_noalloc_matches_workspace_entry_point_and_oracle(cuda, port):
    # Two calls in a row with different sizes: the second reuses the static
    # scratch the first one left behind.  Each is checked against the entry
    # point that takes a caller workspace and against the oracle's
    # CrossEntropyLoss (include/losses.h:34-86).
    for call, (rows, V) in enumerate([(8192, 256), (1000, 300)]):
        r = rng(100 + call)
        logits_h = normal(r, (rows, V), 3.0)
        targets_h = r.integers(0, V, rows)
        logits = torch.as_tensor(logits_h, device="cuda")
        targets = torch.as_tensor(targets_h.astype(np.int32), device="cuda")
        ref_loss, ref_d, ref_err = nk.cross_entropy(logits, targets, denom=rows)
        loss, d, err = noalloc(logits, targets, rows)
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and int(ref_err.item()) == 0
        np.testing.assert_allclose(loss.cpu().numpy(), ref_loss.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(d.cpu().numpy(), ref_d.cpu().numpy(), rtol=RTOL, atol=ATOL)
        o_loss, o_d = port.cross_entropy(logits_h, targets_h.astype(np.float32))
        f_loss, f_d = fp64.cross_entropy(logits_h, targets_h)
        assert_close(loss.cpu().numpy(), np.array([o_loss], np.float32), np.array([f_loss]),
                     what=f"loss call {call}")
        assert_close(d.cpu().numpy(), o_d, f_d, what=f"dlogits call {call}")
