"""Failure path of the bounded device waits, exercised without a GPU fault:
b2q_selftest_stalled_mul_mat launches the GEMM with its TMA producer
withholding every stage, so the consumers' waits run out (after ~2 s); the
kernel drains, frees its tensor memory and returns, the status word carries
the code of the wait that gave up, and the context keeps working."""
import ctypes
import time

import numpy as np
import pytest

import b2q
import oracle as O
from helpers import make_case, rel_frobenius

pytestmark = pytest.mark.gpu

WAIT_CODES = {0x101: "producer", 0x102: "mma", 0x103: "epilogue", 0x104: "drain"}


def test_stalled_gemm_reports_and_recovers(b2q_mod, dev):
    import torch
    M, N, K = 130, 200, 256
    _, wq, x = make_case(11, M, N, K, O.TYPE_Q8_0)
    w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
    x_d = torch.from_numpy(x).to(dev)
    packed = b2q.weight_pack(O.TYPE_Q8_0, w_d, K)
    act = b2q.act_prepare(x_d)
    y = torch.zeros((M, N), dtype=torch.float32, device=dev)
    assert b2q.device_status(clear=True) == 0

    t0 = time.time()
    rc = b2q.lib().b2q_selftest_stalled_mul_mat(packed.data_ptr(), N, K, act.data_ptr(), M, y.data_ptr(),
                                                 N * 4, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    code = ctypes.c_uint(0)
    st = b2q.lib().b2q_device_status(ctypes.byref(code), 1)  # synchronises the device
    elapsed = time.time() - t0
    assert st == 6, "the stalled kernel must report B2Q_ERR_DEVICE"
    assert code.value in WAIT_CODES, hex(code.value)
    assert 1.0 < elapsed < 30.0  # the 2 s budget ran out; nothing hung
    assert torch.count_nonzero(y).item() == 0  # nothing was stored
    assert b2q.device_status(clear=True) == 0  # cleared

    # the context is intact: the same GEMM runs normally afterwards
    out = b2q.mul_mat_prepared(packed, N, K, act, M)
    got = out.cpu().numpy()
    assert rel_frobenius(got, O.mul_mat(O.TYPE_Q8_0, wq, x, O.ACT_X86)) <= 1e-5
    assert b2q.device_status(clear=True) == 0
