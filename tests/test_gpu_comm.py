"""The peer-memory collectives on one GPU: with one rank the fused
all-reduce + RMSNorm is the RMSNorm of h, and its bounded wait gives up
(status word set, the GPU still usable) when a rank's flag never comes: a
two-rank exchange whose second rank does not exist (both table entries point
at this GPU's own buffer, so nothing raises rank 1's flag)."""
import ctypes

import numpy as np
import pytest

from thvm_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _buffer(lib, cols):
    own, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    L.check(lib.sm100_peer_alloc(lib.sm100_comm_bytes(cols), ctypes.byref(own), handle), "peer_alloc")
    return own.value


def test_one_rank_allreduce_is_the_rmsnorm(device):
    import torch
    lib = device.lib
    B, D = 32, 2048
    own = _buffer(lib, D)
    L.check(lib.sm100_comm_set_peers(own, (ctypes.c_void_p * 1)(own), 1), "set_peers")
    rng = np.random.default_rng(0)
    h0 = rng.standard_normal((B, D)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, D).astype(np.float32)
    h, gt = torch.from_numpy(h0).cuda(), torch.from_numpy(g).cuda()
    y = torch.zeros(B, D, dtype=torch.bfloat16, device="cuda")
    for _ in range(3):   # epochs advance; every use sees its own row
        L.check(lib.sm100_comm_allreduce_rmsnorm(h.data_ptr(), gt.data_ptr(), y.data_ptr(), own, 0, 1, B, D, 1e-6,
                                                 0, None), "allreduce_rmsnorm")
    torch.cuda.synchronize()
    assert lib.sm100_comm_status() == 0
    np.testing.assert_array_equal(h.cpu().numpy(), h0)
    ref = h0 / np.sqrt((h0.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * g
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, rtol=2 ** -7, atol=1e-6)
    lib.sm100_peer_free(own)


def test_missing_rank_times_out_with_status(device):
    import torch
    lib = device.lib
    B, D = 2, 64
    own = _buffer(lib, D)
    L.check(lib.sm100_comm_set_peers(own, (ctypes.c_void_p * 2)(own, own), 2), "set_peers")
    h = torch.ones(B, D, device="cuda")
    g = torch.ones(D, device="cuda")
    y = torch.zeros(B, D, dtype=torch.bfloat16, device="cuda")
    lib.sm100_comm_status()
    L.check(lib.sm100_comm_allreduce_rmsnorm(h.data_ptr(), g.data_ptr(), y.data_ptr(), own, 0, 2, B, D, 1e-6, 0,
                                             None), "allreduce_rmsnorm")
    assert lib.sm100_comm_status() != 0   # gave up waiting for rank 1
    assert lib.sm100_comm_status() == 0   # and the word was cleared
    z = torch.arange(8, device="cuda") * 2   # the context still runs work
    assert z.sum().item() == 56
    lib.sm100_peer_free(own)
