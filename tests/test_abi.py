"""CPU checks of the C-ABI library: it loads, and exports every symbol that
include/alb_cuda.h declares.  No compute call is made (no GPU here)."""
import ctypes as C
import subprocess

import pytest

import arclight_b200 as A


def test_library_is_built_and_loads():
    L = A.lib()
    assert L.alb_version() >= 100


def test_every_header_symbol_is_exported():
    syms = A.header_symbols()
    assert len(syms) >= 8
    out = subprocess.run(["nm", "-D", "--defined-only", A.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in syms if s not in exported]
    assert not missing, f"declared in alb_cuda.h but not exported: {missing}"


def test_only_c_abi_symbols_are_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", A.LIB_PATH], capture_output=True, text=True, check=True).stdout
    ours = [l.split()[-1] for l in out.splitlines() if " T " in l]
    leaked = [s for s in ours if not s.startswith("alb_") and not s.startswith("_init") and not s.startswith("_fini")]
    assert not leaked, f"non-ABI symbols exported: {leaked[:10]}"


def test_q4_gpu_layout_sizes():
    L = A.lib()
    # row-interleaved: K/2 nibble bytes + K/32 fp16 scales padded to 8 entries, per row
    assert L.alb_q4_0_row_bytes(2560) == 1280 + 160
    assert L.alb_q4_0_row_bytes(9728) == 4864 + 608
    assert L.alb_q4_0_row_bytes(32) == 16 + 16
    assert L.alb_q4_0_row_bytes(96) == 48 + 16
    assert L.alb_q4_0_row_bytes(33) == 0
    assert L.alb_q4_0_gpu_bytes(9728, 2560) == 9728 * 1440
    assert L.alb_q4_0_gpu_bytes(3, 32) == 256            # rounded up to 256 bytes
    # every row starts 16-byte aligned (one bulk copy per run of rows)
    for k in (32, 96, 1216, 2560, 4096, 9728, 12288):
        assert L.alb_q4_0_row_bytes(k) % 16 == 0


def test_invalid_arguments_are_rejected_without_a_gpu():
    L = A.lib()
    # null pointers / bad K are caught on the host before any CUDA call
    assert L.alb_gemv_q4_0_q8_0(None, None, None, 16, 2560, None, None) == -1
    assert L.alb_mul_mat_q4_0_q8_0(None, None, None, 16, 2560, None) == -1
    dummy16 = 16
    assert L.alb_mul_mat_q4_0_q8_0(dummy16, dummy16, dummy16, 16, 2561, None) == -1   # K % 32
    assert L.alb_gemv_q4_0_q8_0(dummy16, dummy16, dummy16, 16, 12320, None, None) == -1   # K beyond 12288
    assert L.alb_quantize_q8_0(None, None, 33, 1, None) == -1
    assert b"invalid argument" in L.alb_last_error()
    # fused quantizers: n must be a whole number of 32-value blocks
    assert L.alb_rms_norm_q8(None, None, None, None, 1, 2560, 1e-6, None) == -1
    assert L.alb_swiglu_q8(None, None, None, None, 9728, None) == -1
    dummy = 16   # non-null host addresses: the size check fires before any device access
    assert L.alb_rms_norm_q8(dummy, None, None, dummy, 1, 2561, 1e-6, None) == -1
    assert L.alb_swiglu_q8(dummy, dummy, None, dummy, 100, None) == -1
    # communicator: null id / out pointer, bad rank
    assert L.alb_comm_create(None, 0, 1, 0, None) == -1
    assert L.alb_allreduce_sum_f32(None, None, None, 1, None) == -1
    assert L.alb_allgather_f32(None, None, None, 1, None) == -1
    assert L.alb_comm_destroy(None) == 0


def test_set_rows_rejects_bad_shapes_before_any_device_call():
    L = A.lib()
    p = C.c_void_p(4096)   # never dereferenced: the argument checks return first
    assert L.alb_set_rows_f16(p, 2, 1020, p, p, 8, None) == A.ALB_ERR_INVALID    # row_len % 8
    assert L.alb_set_rows_f16(p, 0, 1024, p, p, 8, None) == A.ALB_ERR_INVALID    # no rows
    assert L.alb_set_rows_f16(None, 2, 1024, p, p, 8, None) == A.ALB_ERR_INVALID
    assert L.alb_set_rows_f16(C.c_void_p(4100), 2, 1024, p, p, 8, None) == A.ALB_ERR_INVALID   # unaligned src


def test_headers_are_plain_c_and_the_kv_manager_links(tmp_path):
    """include/*.h compile as C11 (what a cgo / JNI / ctypes binding sees), and a
    C program linked against libalb_cuda.so drives the KV-cache manager (host
    only, no device call): one sequence's cells are its positions."""
    import os
    import shutil
    cc = shutil.which("gcc")
    if not cc:
        pytest.skip("no gcc")
    src = tmp_path / "abi.c"
    src.write_text(r'''
#include <stdio.h>
#include "alb_cuda.h"
#include "alb_kvcache.h"
int main(void) {
    alb_kv_cache * kv = NULL;
    if (alb_kv_create(64, 1, 1, 32, &kv) != ALB_OK) return 1;
    int32_t pos[5] = {0, 1, 2, 3, 4}, seq[5] = {0, 0, 0, 0, 0}, sizes[1] = {5};
    int64_t cells[5];
    uint32_t n_kv = 0;
    if (alb_kv_prepare(kv, sizes, 1, pos, seq, cells) != ALB_OK) return 2;
    if (alb_kv_apply(kv, pos, seq, 5, cells, &n_kv) != ALB_OK || n_kv != 32) return 3;
    for (int i = 0; i < 5; ++i) if (cells[i] != i) return 4;
    if (alb_kv_create(100, 1, 1, 32, &kv) != ALB_ERR_INVALID) return 5;
    printf("ok %s\n", alb_last_error());
    return alb_kv_destroy(kv);
}
''')
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = tmp_path / "abi"
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I" + os.path.join(root, "include"), str(src), "-o", str(exe),
                    "-L" + os.path.dirname(A.LIB_PATH), "-lalb_cuda", "-Wl,-rpath," + os.path.dirname(A.LIB_PATH)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.startswith("ok kv: bad cache shape")
