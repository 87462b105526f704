"""C-ABI checks that need no GPU: the library loads, exports every function
include/b2q.h declares, and rejects bad arguments with status codes before any
device work (fake, never-dereferenced pointers are passed)."""
import ctypes
import os
import subprocess

import pytest

import b2q

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_function(b2q_mod):
    names = b2q.header_functions()
    assert len(names) >= 12, names
    out = subprocess.run(["nm", "-D", "--defined-only", b2q.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # nothing else leaks out of the library under a b2q_ name
    extra = sorted(n for n in exported if n.startswith("b2q_") and n not in names)
    assert not extra, extra


def test_version_and_status_strings(b2q_mod):
    L = b2q.lib()
    assert b"sm_100a" in L.b2q_version()
    for code in range(8):
        assert L.b2q_status_string(code)
    assert L.b2q_status_string(99) == b"unknown status"


def test_size_queries(b2q_mod):
    L = b2q.lib()
    # codes (rounded to 256) + fp32 scales [K/32][round_up(rows, 4)] (rounded to 256)
    assert L.b2q_weight_packed_size(4096, 1024) == 4096 * 1024 + 32 * 4096 * 4
    assert L.b2q_weight_packed_size(10, 64) == 768 + 256
    assert L.b2q_weight_packed_size(10, 33) == 0
    assert L.b2q_mul_mat_workspace_size(1374, 1024, 1024, 1) == \
        1374 * 1024 + ((32 * 1376 * 4 + 255) // 256) * 256
    assert L.b2q_mul_mat_workspace_size(4096, 4096, 1024, 0) == 2 * (4096 * 1024 + 32 * 4096 * 4)
    assert L.b2q_mul_mat_workspace_size(-1, 4, 32, 0) == 0


FAKE = 1 << 20  # aligned, non-null, never dereferenced


@pytest.mark.parametrize("args,expect", [
    # wtype 3 (Q4_1) is not supported
    (dict(wtype=3), b2q.STATUS and 2),
    (dict(k=33), 1),                                    # K not a multiple of 32
    (dict(k=0), 1),
    (dict(n=-1), 1),
    (dict(w=0), 1),                                     # null weight with n > 0
    (dict(ldw=10), 1),                                  # row stride below one row of blocks
    (dict(ldw=1089), 3),                                # odd weight stride
    (dict(w=FAKE + 1), 3),                              # weight not 2-byte aligned
    (dict(x=FAKE + 2), 3),                              # activations not 4-byte aligned
    (dict(ldx=4 * 1024 - 4), 1),                        # x row stride below K floats
    (dict(ldy=4 * 64 + 2), 3),                          # y stride not a multiple of 4
    (dict(variant=5), 1),
    (dict(ws=FAKE + 128), 3),                           # workspace not 256-byte aligned
    (dict(m=1 << 33), 7),                               # beyond int range
])
def test_mul_mat_argument_validation(b2q_mod, args, expect):
    a = dict(wtype=8, w=FAKE, ldw=1088, n=64, k=1024, x=FAKE, m=16, ldx=4096, bias=None,
             y=FAKE, ldy=256, variant=0, ws=FAKE, wsb=1 << 30)
    a.update(args)
    rc = b2q.lib().b2q_mul_mat(a["wtype"], a["w"], a["ldw"], a["n"], a["k"], a["x"], a["m"],
                               a["ldx"], a["bias"], a["y"], a["ldy"], a["variant"], a["ws"],
                               a["wsb"], None)
    assert rc == expect


def test_quantize_argument_validation(b2q_mod):
    L = b2q.lib()
    assert L.b2q_quantize_q8_0(FAKE, 4, 48, 192, FAKE, 34 * 2, 0, None) == 1      # k % 32
    assert L.b2q_quantize_q8_0(FAKE, 4, 64, 128, FAKE, 34, 0, None) == 1          # y stride small
    assert L.b2q_quantize_q8_0(FAKE, 4, 64, 256, FAKE + 1, 68, 0, None) == 3      # odd y
    assert L.b2q_quantize_q8_0(FAKE, 4, 64, 256, FAKE, 68, 2, None) == 1          # variant
    assert L.b2q_quantize_q8_0(None, 4, 64, 256, FAKE, 68, 0, None) == 1          # null x


def test_pack_and_debug_validation(b2q_mod):
    L = b2q.lib()
    assert L.b2q_weight_pack(8, FAKE, 64, 1024, 1088, FAKE, 10, None) == 4       # too small
    assert L.b2q_weight_pack(8, FAKE, 64, 1024, 1088, FAKE + 16, 1 << 24, None) == 3
    assert L.b2q_weight_pack(1, FAKE, 64, 1024, 1088, FAKE, 1 << 24, None) == 2  # F16 weights
    # block-dot debug entry refuses outputs beyond 2^28 dots
    assert L.b2q_block_dots(8, FAKE, 1088, 4096, 1024, FAKE, 4096, 1088, FAKE, FAKE, 1 << 30, None) == 7
    assert L.b2q_mul_mat_q_simt(8, FAKE, 1088, 64, 1024, FAKE, 1 << 20, 1088, FAKE, 256, None) == 7
    code = ctypes.c_uint(0)
    assert L.b2q_device_status(None, 0) == 1


def test_fused_gelu_q8_and_gelu_validation(b2q_mod):
    L = b2q.lib()
    need = L.b2q_act_prepared_size(16, 64)
    f = L.b2q_mul_mat_prepared_gelu_q8
    assert f(FAKE, 48, 1024, FAKE, 16, None, FAKE, 1 << 20, 0, None) == 1        # n % 32
    assert f(FAKE, 64, 1000, FAKE, 16, None, FAKE, 1 << 20, 0, None) == 1        # k % 32
    assert f(FAKE, 64, 1024, FAKE, 16, None, FAKE, 1 << 20, 2, None) == 1        # variant
    assert f(FAKE, 64, 1024, FAKE, 16, None, FAKE + 64, 1 << 20, 0, None) == 3   # act_out alignment
    assert f(FAKE, 64, 1024, FAKE, 16, FAKE + 2, FAKE, 1 << 20, 0, None) == 3    # bias alignment
    assert f(FAKE, 64, 1024, FAKE, 16, None, FAKE, need - 1, 0, None) == 4       # act_out too small
    assert f(FAKE, 64, 1024, FAKE, 16, None, None, 1 << 20, 0, None) == 1        # null act_out
    assert f(FAKE, 64, 1024, FAKE, 1 << 33, None, FAKE, 1 << 40, 0, None) == 7   # beyond int range
    assert f(FAKE, 64, 1024, FAKE, 0, None, FAKE, 0, 0, None) == 0               # m == 0: no-op
    g = L.b2q_gelu
    assert g(FAKE, 4, 8, 16, FAKE, 32, None) == 1                                # x stride < cols
    assert g(FAKE, 4, 8, 32, FAKE, 30, None) == 1                                # y stride < cols
    assert g(FAKE + 2, 4, 8, 32, FAKE, 32, None) == 3
    assert g(FAKE, 4, 8, 34, FAKE, 32, None) == 3                                # stride % 4
    assert g(None, 4, 8, 32, FAKE, 32, None) == 1
    assert g(FAKE, 0, 8, 32, FAKE, 32, None) == 0                                # empty: no-op


def test_norm_modulate_validation(b2q_mod):
    L = b2q.lib()
    f, q = L.b2q_norm_modulate, L.b2q_norm_modulate_q8
    assert f(FAKE, 4, 48, 192, 1e-6, None, None, FAKE, 192, None) == 1            # c % 32
    assert f(FAKE, 4, 8192, 32768, 1e-6, None, None, FAKE, 32768, None) == 7      # c > 4096
    assert f(FAKE, 4, 64, 128, 1e-6, None, None, FAKE, 256, None) == 1            # x stride < c
    assert f(FAKE, 4, 64, 256, -1.0, None, None, FAKE, 256, None) == 1            # eps < 0
    assert f(FAKE + 4, 4, 64, 256, 1e-6, None, None, FAKE, 256, None) == 3        # x not 16-byte aligned
    assert f(FAKE, 4, 64, 260, 1e-6, None, None, FAKE, 256, None) == 3            # stride % 16
    assert f(FAKE, 4, 64, 256, 1e-6, FAKE + 4, None, FAKE, 256, None) == 3        # scale alignment
    assert f(FAKE, 4, 64, 256, 1e-6, None, None, None, 256, None) == 1            # null y
    assert f(FAKE, 4, 64, 256, 1e-6, None, None, FAKE + 8, 256, None) == 3        # y alignment
    assert f(FAKE, 0, 64, 256, 1e-6, None, None, FAKE, 256, None) == 0            # empty: no-op
    need = L.b2q_act_prepared_size(4, 64)
    assert q(FAKE, 4, 64, 256, 1e-6, None, None, 2, FAKE, need, None) == 1        # variant
    assert q(FAKE, 4, 64, 256, 1e-6, None, None, 0, FAKE + 16, need, None) == 3   # act alignment
    assert q(FAKE, 4, 64, 256, 1e-6, None, None, 0, FAKE, need - 1, None) == 4    # act too small
    assert q(FAKE, 0, 64, 256, 1e-6, None, None, 0, FAKE, 0, None) == 0


def test_gate_residual_validation(b2q_mod):
    f = b2q.lib().b2q_mul_mat_prepared_gate_residual
    assert f(FAKE, 64, 1000, FAKE, 16, None, None, FAKE, 256, FAKE, 256, None) == 1         # k % 32
    assert f(FAKE, 64, 1024, FAKE, 16, None, None, None, 256, FAKE, 256, None) == 1         # null resid
    assert f(FAKE, 64, 1024, FAKE, 16, None, None, FAKE, 128, FAKE, 256, None) == 1         # resid stride
    assert f(FAKE, 64, 1024, FAKE, 16, None, None, FAKE, 512, FAKE, 256, None) == 1         # aliased, strides differ
    assert f(FAKE, 64, 1024, FAKE, 16, None, FAKE + 1, FAKE + 4096, 256, FAKE, 256, None) == 3  # gate alignment
    assert f(FAKE, 64, 1024, FAKE, 0, None, None, FAKE, 256, FAKE, 256, None) == 0          # m == 0


def test_weight_upload_validation(b2q_mod):
    f = b2q.lib().b2q_weight_upload
    big = 1 << 24
    assert f(1, FAKE, 64, 1024, 1088, FAKE, big, FAKE, big, None) == 2            # F16 weights
    assert f(8, FAKE, 64, 1000, 1088, FAKE, big, FAKE, big, None) == 1            # k % 32
    assert f(8, FAKE, 64, 1024, 1000, FAKE, big, FAKE, big, None) == 1            # row stride < row
    assert f(8, FAKE, 64, 1024, 1088, None, big, FAKE, big, None) == 1            # null staging
    assert f(8, FAKE, 64, 1024, 1088, FAKE, 1087, FAKE, big, None) == 4           # staging < one row
    assert f(8, FAKE, 64, 1024, 1088, FAKE, big, FAKE, 10, None) == 4             # packed too small
    assert f(8, FAKE, 64, 1024, 1088, FAKE, big, FAKE + 16, big, None) == 3       # packed alignment
    assert f(8, FAKE, 0, 1024, 1088, FAKE, 0, FAKE, 0, None) == 0                 # n == 0: no-op


def test_empty_shapes_are_noops_without_device(b2q_mod):
    L = b2q.lib()
    # m == 0 or n == 0: validated, nothing launched, OK even without a GPU
    assert L.b2q_mul_mat(8, FAKE, 1088, 64, 1024, FAKE, 0, 4096, None, FAKE, 256, 0, FAKE, 0, None) == 0
    assert L.b2q_mul_mat_packed(FAKE, 0, 1024, FAKE, 16, 4096, None, FAKE, 0, 0, FAKE, 0, None) == 0


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "b2q.h"\nint main(void){return b2q_status_string(0)==0;}\n')
    r = subprocess.run(["/usr/bin/gcc", "-std=c99", "-Wall", "-Werror", "-c",
                        "-I", os.path.join(REPO, "include"), str(src), "-o", str(tmp_path / "t.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_q4_k_validation(b2q_mod):
    L = b2q.lib()
    # typed sizes: Q4_K packs as its own rows; Q8_K is the codes plus one fp32 scale per 256 values
    assert L.b2q_weight_packed_bytes(12, 64, 1024) == 64 * 4 * 144                 # the rows themselves
    assert L.b2q_weight_packed_bytes(8, 64, 1024) == L.b2q_weight_packed_size(64, 1024)
    assert L.b2q_weight_packed_bytes(12, 64, 96) == 0 and L.b2q_weight_packed_bytes(3, 64, 1024) == 0
    assert L.b2q_act_prepared_bytes(2, 5, 512) == 5 * 512 + 256            # codes, then d [2][8] padded to 256
    assert L.b2q_act_prepared_bytes(2, 4, 96) == 0 and L.b2q_act_prepared_bytes(0, 4, 96) == L.b2q_act_prepared_size(4, 96)
    assert L.b2q_mul_mat_workspace_bytes(12, 4, 64, 1024, 1) == L.b2q_act_prepared_bytes(2, 4, 1024)
    big = 1 << 30
    # raw Q4_K: k % 256, the variant must be Q8_K and Q8_K only goes with Q4_K
    assert L.b2q_mul_mat(12, FAKE, 144 * 4, 64, 288, FAKE, 4, 4096, None, FAKE, 256, 2, FAKE, big, None) == 1
    assert L.b2q_mul_mat(12, FAKE, 144 * 4, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 0, FAKE, big, None) == 1
    assert L.b2q_mul_mat(8, FAKE, 1088, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 2, FAKE, big, None) == 1
    assert L.b2q_mul_mat(12, FAKE, 144 * 3, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 2, FAKE, big, None) == 1
    # pack: the buffer must hold the rows
    assert L.b2q_weight_pack(12, FAKE, 64, 1024, 576, FAKE, L.b2q_weight_packed_bytes(12, 64, 1024) - 1, None) == 4
    f = L.b2q_mul_mat_prepared_q4_k
    assert f(FAKE, 64, 1000, FAKE, 4, None, None, None, 0, FAKE, 256, None) == 1   # k % 256
    assert f(FAKE, 64, 1024, FAKE, 4, None, None, None, 0, FAKE, 128, None) == 1   # y stride
    assert f(FAKE, 64, 1024, FAKE + 16, 4, None, None, None, 0, FAKE, 256, None) == 3
    assert f(FAKE, 64, 1024, FAKE, 4, None, None, FAKE, 512, FAKE, 256, None) == 1  # aliased, strides differ
    assert f(FAKE, 64, 1024, FAKE, 0, None, None, None, 0, FAKE, 256, None) == 0
    # debug check paths are for the 32-value block types
    assert L.b2q_block_dots(12, FAKE, 576, 64, 1024, FAKE, 4, 1088, FAKE, FAKE, big, None) == 2
    assert L.b2q_mul_mat_q_simt(12, FAKE, 576, 64, 1024, FAKE, 4, 1088, FAKE, 256, None) == 2
    # Q8_K activations: k % 256; the fused GELU quantize does not produce Q8_K
    assert L.b2q_act_prepare(FAKE, 4, 96, 384, 2, FAKE, big, None) == 1
    assert L.b2q_mul_mat_prepared_gelu_q8(FAKE, 256, 1024, FAKE, 4, None, FAKE, big, 2, None) == 1


def test_attention_io_validation(b2q_mod):
    L = b2q.lib()
    qkv, r2h, hq, ln = L.b2q_qkv_heads, L.b2q_rows_to_heads, L.b2q_heads_act_prepare, L.b2q_layer_norm_q8
    st = 3 * 4 * 64 * 4
    assert qkv(FAKE, 2, 8, 4, 48, st, None, None, 1e-6, FAKE, FAKE, FAKE, None) == 1     # D not 32/64/128
    assert qkv(FAKE, 2, 8, 4, 64, st - 4, None, None, 1e-6, FAKE, FAKE, FAKE, None) == 1  # stride < 3C
    assert qkv(FAKE, 0, 8, 4, 64, st, None, None, 1e-6, FAKE, FAKE, FAKE, None) == 0     # empty: no-op
    assert r2h(FAKE, 2, 8, 4, 64, 3, 4 * 64 * 8, FAKE, FAKE, None) == 1                  # parts > 2
    assert r2h(FAKE, 2, 8, 4, 64, 2, 4 * 64 * 8, FAKE, None, None) == 1                  # parts 2, null out1
    assert r2h(FAKE, 2, 8, 4, 64, 2, 4 * 64 * 8 - 4, FAKE, FAKE, None) == 1              # stride < 2C
    assert r2h(FAKE + 2, 2, 8, 4, 64, 1, 4 * 64 * 4, FAKE, None, None) == 3              # src alignment
    assert r2h(FAKE, 2, 8, 4, 64, 1, 4 * 64 * 4, FAKE + 1, None, None) == 3              # out alignment
    assert r2h(FAKE, 0, 8, 4, 64, 1, 4 * 64 * 4, FAKE, None, None) == 0                  # empty: no-op
    mh = L.b2q_mul_mat_prepared_heads_f16
    assert mh(FAKE, 512, 256, FAKE, 32, None, 2, 16, 4, 64, 3, FAKE, FAKE, None) == 1     # parts > 2
    assert mh(FAKE, 512, 256, FAKE, 32, None, 2, 16, 4, 64, 2, FAKE, None, None) == 1     # parts 2, null out1
    assert mh(FAKE, 500, 256, FAKE, 32, None, 2, 16, 4, 64, 2, FAKE, FAKE, None) == 1     # n != parts*H*D
    assert mh(FAKE, 512, 256, FAKE, 30, None, 2, 16, 4, 64, 2, FAKE, FAKE, None) == 1     # m != B*T
    assert mh(FAKE, 256, 256, FAKE, 32, None, 2, 16, 8, 32, 1, FAKE, None, None) == 2     # D != 64
    assert mh(FAKE, 512, 256, FAKE, 8, None, 2, 4, 4, 64, 2, FAKE, FAKE, None) == 2       # few tokens
    assert mh(FAKE + 16, 512, 256, FAKE, 32, None, 2, 16, 4, 64, 2, FAKE, FAKE, None) == 3  # weight alignment
    assert mh(FAKE, 512, 256, FAKE, 32, None, 2, 16, 4, 64, 2, FAKE + 1, FAKE, None) == 3  # out alignment
    assert mh(FAKE, 512, 256, FAKE, 0, None, 0, 16, 4, 64, 2, FAKE, FAKE, None) == 0      # empty: no-op
    need = L.b2q_act_prepared_size(16, 256)
    assert hq(FAKE, 2, 8, 4, 48, 0, 0, 0, 0, FAKE, need, None) == 1                       # D % 32
    assert hq(FAKE, 2, 8, 4, 64, -1, 0, 0, 0, FAKE, need, None) == 1                      # negative stride
    assert hq(FAKE, 2, 8, 4, 64, 0, 0, 0, 0, FAKE + 16, need, None) == 3                  # act alignment
    assert hq(FAKE, 2, 8, 4, 64, 0, 0, 0, 0, FAKE, need - 1, None) == 4                   # act too small
    need = L.b2q_act_prepared_size(4, 64)
    assert ln(FAKE, 4, 48, 192, 1e-6, None, None, 0, FAKE, need, None) == 1              # c % 32
    assert ln(FAKE, 4, 64, 256, 1e-6, FAKE + 4, None, 0, FAKE, need, None) == 3          # weight alignment
    assert ln(FAKE, 4, 64, 256, 1e-6, None, None, 2, FAKE, need, None) == 1              # variant
    assert ln(FAKE, 4, 64, 256, 1e-6, None, None, 0, FAKE, need - 1, None) == 4          # act too small
    assert ln(FAKE, 0, 64, 256, 1e-6, None, None, 0, FAKE, 0, None) == 0                 # empty: no-op


def test_f16_validation(b2q_mod):
    L = b2q.lib()
    f = L.b2q_mul_mat
    ws = 1 << 22
    assert L.b2q_mul_mat_workspace_bytes(1, 33, 65, 256, 0) == (33 * 256 * 2 + 255) // 256 * 256
    assert L.b2q_mul_mat_workspace_bytes(1, 33, 65, 252, 0) == 0                              # k % 8
    assert f(1, FAKE, 2016, 64, 1004, FAKE, 4, 4016, None, FAKE, 256, 0, FAKE, ws, None) == 1  # k % 8
    assert f(1, FAKE, 1024, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 0, FAKE, ws, None) == 1  # row stride < 2k
    assert f(1, FAKE + 2, 2048, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 0, FAKE, ws, None) == 3  # w alignment
    assert f(1, FAKE, 2056, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 0, FAKE, ws, None) == 3  # stride % 16
    assert f(1, FAKE, 2048, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 2, FAKE, ws, None) == 1  # Q8_K variant
    assert f(1, FAKE, 2048, 64, 1024, FAKE, 4, 4096, None, FAKE, 256, 0, FAKE, 100, None) == 4  # workspace
    assert f(1, FAKE, 2048, 64, 1024, FAKE, 0, 4096, None, FAKE, 256, 0, FAKE, 0, None) == 0    # m == 0


def test_sparse_validation(b2q_mod):
    L = b2q.lib()
    conv, sm = L.b2q_sparse_conv_f16, L.b2q_sparse_scatter_mean_f16
    ws = 1 << 24
    assert L.b2q_sparse_conv_f16_workspace_bytes(10, 12, 16) == 0                          # C % 8
    assert L.b2q_sparse_conv_f16_workspace_bytes(10, 8, 16) == 4352 + 256                  # 10*27*8*2 -> 4352
    assert conv(FAKE, 10, 12, FAKE, 16, None, FAKE, FAKE, FAKE, ws, None) == 1             # C % 8
    assert conv(FAKE + 8, 10, 8, FAKE, 16, None, FAKE, FAKE, FAKE, ws, None) == 3          # x alignment
    assert conv(FAKE, 10, 8, FAKE, 16, FAKE + 1, FAKE, FAKE, FAKE, ws, None) == 3          # bias alignment
    assert conv(FAKE, 10, 8, FAKE, 16, None, FAKE, FAKE, FAKE, 100, None) == 4             # workspace
    assert conv(FAKE, 0, 8, FAKE, 16, None, FAKE, FAKE, FAKE, 0, None) == 0                # no tokens
    assert L.b2q_sparse_scatter_mean_workspace_bytes(100, 10) == 768                       # (31 + 100) * 4 -> 768
    assert sm(FAKE, 100, 12, FAKE, FAKE, 10, FAKE, FAKE, ws, None) == 1                    # C % 8
    assert sm(FAKE, 100, 8, FAKE, FAKE, 10, FAKE + 4, FAKE, ws, None) == 3                 # out alignment
    assert sm(FAKE, 100, 8, FAKE, FAKE, 10, FAKE, FAKE, 100, None) == 4                    # workspace
    assert sm(FAKE, 100, 8, FAKE, FAKE, 0, FAKE, FAKE, 0, None) == 0                       # no coarse rows
    plan, run = L.b2q_sparse_scatter_plan, L.b2q_sparse_scatter_mean_f16_planned
    assert plan(FAKE, 100, 10, FAKE, 100, None) == 4                                       # plan too small
    assert plan(FAKE + 2, 100, 10, FAKE, ws, None) == 3                                    # rows alignment
    assert plan(FAKE, 100, 0, FAKE, 0, None) == 0                                          # no coarse rows
    assert run(FAKE, 100, 12, FAKE, FAKE, 10, FAKE, None) == 1                             # C % 8
    assert run(FAKE, 100, 8, None, FAKE, 10, FAKE, None) == 1                              # no plan


def test_sparse_conv_plan_validation(b2q_mod):
    L = b2q.lib()
    plan, run = L.b2q_sparse_conv_plan, L.b2q_sparse_conv_f16_planned
    ws = 1 << 26
    assert L.b2q_sparse_conv_plan_bytes(100) > 27 * 100 * 4
    assert L.b2q_sparse_conv_f16_planned_workspace_bytes(100, 96, 64) == 0                 # C % 64
    assert L.b2q_sparse_conv_f16_planned_workspace_bytes(100, 64, 60) == 0                 # Cout % 8
    assert plan(FAKE, 100, FAKE, 100, None) == 4                                           # plan too small
    assert plan(FAKE + 2, 100, FAKE, ws, None) == 3                                        # index alignment
    assert run(FAKE, 100, 96, FAKE, 64, None, FAKE, FAKE, FAKE, ws, None) == 1             # C % 64
    assert run(FAKE, 100, 64, FAKE, 60, None, FAKE, FAKE, FAKE, ws, None) == 1             # Cout % 8
    assert run(FAKE, 100, 64, FAKE, 64, None, FAKE, FAKE + 8, FAKE, ws, None) == 3         # y alignment
    assert run(FAKE, 100, 64, FAKE, 64, None, FAKE, FAKE, FAKE, 100, None) == 4            # workspace
    assert run(FAKE, 0, 64, FAKE, 64, None, FAKE, FAKE, FAKE, 0, None) == 0                # no tokens
