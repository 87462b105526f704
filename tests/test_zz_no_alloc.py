"""b2q_mul_mat_packed_noalloc (activations in the library's fixed device array)
against b2q_mul_mat_packed (activations in a caller workspace), through the C ABI.

Collected last on purpose: the GPU case must pass in a fresh process and after
every other test has used the library."""
import ctypes

import numpy as np
import pytest

import b2q
import oracle as O
from helpers import make_case, rel_frobenius

RTOL = 1e-5  # relative Frobenius tolerance of the fp32 result


def test_noalloc_rejects_sizes_beyond_its_array(b2q_mod):
    # Returns before any CUDA call, so it runs without a device.
    k = 4096
    m = b2q.NOALLOC_SCRATCH_BYTES // k  # codes alone fill the array; the scales do not fit
    assert b2q.act_prepared_size(m, k) > b2q.NOALLOC_SCRATCH_BYTES
    rc = b2q.lib().b2q_mul_mat_packed_noalloc(None, 64, k, None, m, k * 4, None, None, 64 * 4,
                                              b2q.ACT_X86, None)
    assert rc == 7  # B2Q_ERR_TOO_LARGE
    rc = b2q.lib().b2q_mul_mat_packed_noalloc(None, 64, 100, None, 4, 400, None, None, 256,
                                              b2q.ACT_X86, None)
    assert rc == 1  # k % 32 != 0


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_on_consecutive_calls(b2q_mod, dev):
    import torch
    cases = [  # (seed, M, N, K, wtype): the second call is smaller, over the first's leftovers
        (31, 1374, 384, 1024, O.TYPE_Q4_0),
        (32, 300, 200, 640, O.TYPE_Q8_0),
    ]
    for seed, M, N, K, wtype in cases:
        _, wq, x = make_case(seed, M, N, K, wtype)
        w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
        x_d = torch.from_numpy(x).to(dev)
        packed = b2q.weight_pack(wtype, w_d, K)
        y_ws = b2q.mul_mat_packed(packed, N, K, x_d)
        y_na = b2q.mul_mat_packed_noalloc(packed, N, K, x_d)
        torch.cuda.synchronize()
        a, b = y_na.cpu().numpy(), y_ws.cpu().numpy()
        assert np.isfinite(a).all()
        assert rel_frobenius(a, b) <= RTOL
    code = ctypes.c_uint(0)
    assert b2q.lib().b2q_device_status(ctypes.byref(code), 1) == 0 and code.value == 0
