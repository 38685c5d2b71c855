"""Bounded device waits: a fused-collective kernel whose peer never signals gives up after about a
second, records an error code the host reads, and leaves the CUDA context usable. The missing peer
is a flag slot that nothing writes (both "ranks" are this process); no GPU fault is involved."""
import time

import pytest
import torch

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu

K_ERR_COMM_WAIT = 3


def test_comm_wait_expires_with_error_status(cuda_ext):
    T, H = 4, 256
    dev = "cuda"
    data = torch.randn(T, H, device=dev)
    flags = torch.zeros(256 * 8, dtype=torch.int32, device=dev)
    epochs = torch.zeros(256, dtype=torch.int32, device=dev)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    resid = torch.zeros(T, H, device=dev)
    w = torch.ones(H, device=dev)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    t0 = time.time()
    ops.C().ar_add_rmsnorm([data.data_ptr()] * 2, [flags.data_ptr()] * 2, epochs, 0, T, H, 1, 0, resid, w, 1e-5,
                           out, err, 148)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(err[0]) == K_ERR_COMM_WAIT
    assert dt < 20
    # the context is still usable: a normal kernel runs and is correct
    r = torch.randn(T, H, device=dev)
    want = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + 1e-5)
    o = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ops.add_rmsnorm(r, w, T, H, 1e-5, out=o)
    torch.cuda.synchronize()
    assert (o.float() - want).abs().max().item() < 0.05
