"""b2q_mul_mat_packed_noalloc (activations in the library's fixed device array)
against b2q_mul_mat_packed (activations in a caller workspace), through the C ABI.

The no-allocation entry serves callers that cannot call cudaMalloc: a ggml
backend computing a graph whose buffers are already placed, or a serving loop
that must not synchronise the device.  It runs the same kernels on the same
bytes as the workspace entry, so its outputs must be equal bit for bit.

Collected last on purpose, so a run that stops at the first failure has run
every other test first.  The GPU cases cover both orders: in the pytest process
after every other test has used the library, and in a fresh process where the
first no-allocation call (after packing its weight) runs the per-device set-up."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import b2q
import oracle as O
from helpers import make_case

TOO_LARGE, INVALID_ARG = 7, 1


def test_noalloc_rejects_sizes_beyond_its_array(b2q_mod):
    # Every rejection returns before any CUDA call, so it runs without a device.
    L = b2q.lib()
    limit = b2q.NOALLOC_SCRATCH_BYTES
    # Q8_0 activations: the codes alone fill the array, the scales do not fit.
    k = 4096
    m = limit // k
    assert L.b2q_act_prepared_bytes(b2q.ACT_X86, m, k) > limit
    assert L.b2q_mul_mat_packed_noalloc(None, 64, k, None, m, k * 4, None, None, 256, b2q.ACT_X86, None) == TOO_LARGE
    assert L.b2q_mul_mat_packed_noalloc(None, 64, 100, None, 4, 400, None, None, 256, b2q.ACT_X86, None) == INVALID_ARG
    # Q8_K activations (Q4_K weights): the largest m that fits, and one row more.
    k = 2048
    lo, hi = 1, limit // k + 1  # the size at lo fits, the size at hi does not
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if L.b2q_act_prepared_bytes(b2q.ACT_Q8_K, mid, k) <= limit else (lo, mid)
    m_fit = lo
    assert L.b2q_act_prepared_bytes(b2q.ACT_Q8_K, m_fit + 1, k) > limit
    assert L.b2q_mul_mat_packed_noalloc(None, 64, k, None, m_fit + 1, k * 4, None, None, 256,
                                        b2q.ACT_Q8_K, None) == TOO_LARGE
    # An unknown variant is an invalid argument whatever the size.
    assert L.b2q_mul_mat_packed_noalloc(None, 64, 4096, None, limit // 4096, 4096 * 4, None, None, 256,
                                        7, None) == INVALID_ARG
    # Q8_K needs k % 256 == 0.
    assert L.b2q_mul_mat_packed_noalloc(None, 64, 96, None, 4, 384, None, None, 256,
                                        b2q.ACT_Q8_K, None) == INVALID_ARG


def _compare_consecutive_calls(dev):
    """Two calls in a row per case (the second over the first's leftovers in the
    shared array), each equal bit for bit to the workspace entry."""
    import torch
    cases = [  # (seed, M, N, K, wtype, variant)
        (31, 1374, 384, 1024, O.TYPE_Q4_0, b2q.ACT_X86),
        (32, 300, 200, 640, O.TYPE_Q8_0, b2q.ACT_REF),
        (33, 517, 256, 1024, O.TYPE_Q4_K, b2q.ACT_Q8_K),
        (34, 77, 96, 512, O.TYPE_Q8_0, b2q.ACT_X86),
    ]
    for seed, M, N, K, wtype, variant in cases:
        rng = np.random.default_rng(seed)
        if wtype == O.TYPE_Q4_K:
            wq = O.random_q4_k(N, K, seed=seed)
            x = rng.standard_normal((M, K)).astype(np.float32)
        else:
            _, wq, x = make_case(seed, M, N, K, wtype)
        w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
        x_d = torch.from_numpy(x).to(dev)
        bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
        packed = b2q.weight_pack(wtype, w_d, K)
        y_ws = b2q.mul_mat_packed(packed, N, K, x_d, bias=bias, variant=variant)
        y_na = b2q.mul_mat_packed_noalloc(packed, N, K, x_d, bias=bias, variant=variant)
        torch.cuda.synchronize()
        a, b = y_na.cpu().numpy(), y_ws.cpu().numpy()
        assert np.isfinite(a).all()
        assert np.array_equal(a, b), f"case {seed}: no-allocation output differs from the workspace entry"
    code = ctypes.c_uint(0)
    assert b2q.lib().b2q_device_status(ctypes.byref(code), 1) == 0 and code.value == 0


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_on_consecutive_calls(b2q_mod, dev):
    _compare_consecutive_calls(dev)


@pytest.mark.gpu
def test_noalloc_first_call_in_a_fresh_process(b2q_mod, dev):
    """A new process whose first no-allocation call runs the set-up (the weight
    is packed just before it), then two calls compared with the workspace entry."""
    here = os.path.dirname(os.path.abspath(__file__))
    code = (
        "import sys, numpy as np, torch\n"
        f"sys.path[:0] = {[here, os.path.join(os.path.dirname(here), 'sam-3d-objects-ggml_b200'), os.path.join(os.path.dirname(here), 'oracle')]!r}\n"
        "import b2q, oracle as O\n"
        "from helpers import make_case\n"
        "dev = torch.device('cuda:0')\n"
        "_, wq, x = make_case(35, 200, 128, 512, O.TYPE_Q8_0)\n"
        "w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)\n"
        "x_d = torch.from_numpy(x).to(dev)\n"
        "packed = b2q.weight_pack(O.TYPE_Q8_0, w_d, 512)\n"
        "y_na = b2q.mul_mat_packed_noalloc(packed, 128, 512, x_d)\n"
        "y_na2 = b2q.mul_mat_packed_noalloc(packed, 128, 512, x_d)\n"
        "y_ws = b2q.mul_mat_packed(packed, 128, 512, x_d)\n"
        "torch.cuda.synchronize()\n"
        "assert torch.equal(y_na, y_ws) and torch.equal(y_na2, y_ws)\n"
        "print('fresh-process no-allocation call: equal')\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
