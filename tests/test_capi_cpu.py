"""C ABI checks that need no GPU: the library loads, exports every symbol the
public headers declare, and rejects bad arguments with the documented status
before touching a device."""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

from leankv_b200 import _lib as L


def test_library_builds_and_loads():
    from leankv_b200 import build
    build.build()
    lib = L.load()
    assert lib.tq_abi_version() == 1


def test_every_header_symbol_is_exported():
    names = L.header_functions()
    # the ggml drop-ins plus the tq_* API must all be declared
    for n in ("quantize_row_tq3_0_ref", "quantize_row_tq4_0_ref", "dequantize_row_tq3_0", "dequantize_row_tq4_0",
              "quantize_row_tq3_0", "quantize_row_tq4_0", "hadamard_transform", "hadamard_transform_row",
              "tq_quantize_cuda", "tq_dequantize_cuda", "tq_hadamard_cuda"):
        assert n in names
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_every_header_symbol_has_a_python_signature():
    missing = [n for n in L.header_functions() if n not in L.SIGNATURES]
    assert not missing, missing


def test_header_compiles_as_c_and_cpp(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "leankv_tq.h"\nint main(void){ return (int)sizeof(block_tq4_0) - 18 + (int)sizeof(block_tq3_0) - 14; }\n')
    for cc, ext in (("gcc", "c"), ("g++", "cpp")):
        f = tmp_path / f"t.{ext}"
        f.write_text(src.read_text())
        exe = tmp_path / f"t_{ext}"
        subprocess.run([cc, "-std=c11" if ext == "c" else "-std=c++17", "-I", L.HEADER_DIR, str(f), "-o", str(exe)],
                       check=True)
        assert subprocess.run([str(exe)]).returncode == 0


@pytest.mark.parametrize("call,status", [
    (lambda lib: lib.tq_quantize_cuda(4, None, 0, None, 33, 0, 0, None), 1),        # k % 32
    (lambda lib: lib.tq_quantize_cuda(5, None, 0, None, 32, 0, 0, None), 1),        # bad type
    (lambda lib: lib.tq_quantize_cuda(4, None, 7, None, 32, 0, 0, None), 1),        # bad dtype
    (lambda lib: lib.tq_quantize_cuda(4, None, 0, None, 32, 0, 0, None), 1),        # null pointers
    (lambda lib: lib.tq_quantize_cuda(4, 16, 0, 16, 32, 0, 2, None), 2),            # opt rounding on TQ4
    (lambda lib: lib.tq_quantize_cuda(3, 16, 0, 16, 96, 48, 0, None), 1),           # head_dim not pow2
    (lambda lib: lib.tq_quantize_cuda(3, 16, 0, 16, 4096, 2048, 0, None), 2),       # fused FWHT > 1024
    (lambda lib: lib.tq_quantize_cuda(3, 18, 0, 16, 64, 0, 0, None), 3),            # x misaligned for f32
    (lambda lib: lib.tq_dequantize_cuda(4, 16, 18, 0, 64, None), 3),                # y misaligned
    (lambda lib: lib.tq_hadamard_cuda(16, 96, 64, None), 1),                        # n % head_dim
    (lambda lib: lib.tq_hadamard_cuda(16, 1 << 17, 1 << 16, None), 2),              # head_dim > 32768
    (lambda lib: lib.tq_quantize_host(4, None, 0, None, 31, 0, 0), 1),
])
def test_argument_errors(call, status):
    lib = L.load()
    assert call(lib) == status
    assert lib.tq_last_error_string()  # a message is set


def test_tq21_argument_errors_and_layout(tmp_path):
    """TQ2_1 entry points check k and pointers before any device work; block_tq2_1 is 44 bytes
    with the TQ3_0 sub-block first (runs without a GPU)."""
    lib = L.load()
    assert lib.tq_quantize_tq2_1_cuda(16, 0, 16, 96, None) == 1          # k not a multiple of 128
    assert lib.tq_quantize_tq2_1_cuda(16, 7, 16, 128, None) == 1         # bad dtype
    assert lib.tq_quantize_tq2_1_cuda(None, 0, None, 128, None) == 1     # null pointers
    assert lib.tq_quantize_tq2_1_cuda(None, 0, None, 0, None) == 0       # nothing to do
    assert lib.tq_dequantize_tq2_1_cuda(16, 16, 130, None) == 1
    assert lib.tq_dequantize_tq2_1_cuda(17, 16, 128, None) == 3          # blocks not 2-byte aligned
    src = tmp_path / "b.c"
    src.write_text('#include "leankv_tq.h"\n#include <stddef.h>\n'
                   'int main(void){ return sizeof(block_tq2_1) != 44 || offsetof(block_tq2_1, d_n0) != 14 ||'
                   ' offsetof(block_tq2_1, d_n2) != 34; }\n')
    exe = tmp_path / "b"
    subprocess.run(["gcc", "-I", L.HEADER_DIR, str(src), "-o", str(exe)], check=True)
    assert subprocess.run([str(exe)]).returncode == 0


def test_zero_length_is_a_noop():
    lib = L.load()
    assert lib.tq_quantize_cuda(4, None, 0, None, 0, 0, 0, None) == 0
    assert lib.tq_dequantize_cuda(3, None, None, 0, 0, None) == 0


def test_status_strings():
    lib = L.load()
    for s in range(8):
        assert lib.tq_status_string(s)


def test_dropin_aborts_like_reference_assert():
    """k % 32 != 0 aborts (the reference asserts) — checked in a child process."""
    code = ("import ctypes, numpy as np\n"
            f"lib = ctypes.CDLL({L.LIB_PATH!r})\n"
            "x = np.zeros(33, np.float32); y = np.zeros(64, np.uint8)\n"
            "lib.quantize_row_tq4_0_ref(ctypes.c_void_p(x.ctypes.data), ctypes.c_void_p(y.ctypes.data), ctypes.c_int64(33))\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode != 0
    assert "k % 32" in r.stderr


def test_ops_reject_cpu_tensors():
    import torch
    from leankv_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.quantize(torch.zeros(64), 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.dequantize(torch.zeros(18, dtype=torch.uint8), 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.hadamard_(torch.zeros(64), 64)


def test_attention_argument_errors():
    """The attention entry point validates its argument block before any device work."""
    import torch
    from leankv_b200 import attention as A
    lib = A._bind()
    a = A.AttnArgs()
    a.batch, a.n_q_heads, a.n_kv_heads, a.head_dim = 1, 12, 8, 128          # 12 % 8 != 0
    a.k_type = a.v_type = 4
    a.kv_capacity = 64
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 1
    a.n_q_heads = 72                                                         # group 9
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 2
    a.n_q_heads = 64                                                         # group 8 ok, head_dim 64 not
    a.head_dim = 64
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 2
    a.head_dim = 128
    a.kv_capacity = 63                                                       # odd capacity
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 1
    a.kv_capacity = 64
    a.q = a.out = 16
    a.k_cache = 24                                                           # not 16-byte aligned
    a.v_cache = 32
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 3
    a.k_cache = 32
    assert lib.tq_decode_attention_workspace_size(C.byref(a)) > 0
    assert lib.tq_decode_attention_cuda(C.byref(a), None) == 1               # no workspace
    assert ctypes_sizeof_matches_c()


def ctypes_sizeof_matches_c(tmp=None):
    """sizeof(tq_decode_attention_args) in C equals the ctypes mirror."""
    import tempfile
    from leankv_b200 import attention as A
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "s.c")
        open(src, "w").write('#include "leankv_tq.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                             'int main(void){printf("%zu %zu %zu\\n", sizeof(tq_decode_attention_args),'
                             ' offsetof(tq_decode_attention_args, workspace_bytes),'
                             ' offsetof(tq_decode_attention_args, sm_scale)); return 0;}\n')
        exe = os.path.join(td, "s")
        subprocess.run(["gcc", "-I", L.HEADER_DIR, src, "-o", exe], check=True)
        sz, off_ws, off_sc = map(int, subprocess.run([exe], capture_output=True, text=True).stdout.split())
    return (sz == C.sizeof(A.AttnArgs) and off_ws == A.AttnArgs.workspace_bytes.offset
            and off_sc == A.AttnArgs.sm_scale.offset)


def test_paged_argument_errors():
    """The paged attention and append entry points check the page description before any
    device work (runs without a GPU)."""
    from leankv_b200 import attention as A
    lib = A._bind()
    a = A.AttnArgs()
    a.batch, a.n_q_heads, a.n_kv_heads, a.head_dim = 2, 16, 2, 128
    a.k_type = a.v_type = 4
    a.q = a.out = 16
    a.k_cache = a.v_cache = 32
    table = (C.c_int32 * 8)()
    pg = A.KVPages()
    pg.page_table = C.addressof(table)
    pg.max_pages_per_seq, pg.num_pages, pg.page_size = 4, 8, 16
    a.kv_capacity = 64
    assert lib.tq_decode_attention_paged_cuda(C.byref(a), None, None) == 1            # no page description
    assert lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), None) == 1     # no workspace
    for field, bad in (("page_size", 24), ("page_size", 8), ("num_pages", 0), ("max_pages_per_seq", 0)):
        saved = getattr(pg, field)
        setattr(pg, field, bad)
        assert lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), None) == 1, field
        setattr(pg, field, saved)
    a.kv_capacity = 62                                                                 # != 4 pages x 16
    assert lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), None) == 1
    a.kv_capacity = 64
    pg.page_table = None
    assert lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), None) == 1      # null table
    a.batch = 0
    assert lib.tq_decode_attention_paged_cuda(C.byref(a), C.byref(pg), None) == 0      # nothing to do
    lib2 = L.load()
    pg.page_table = C.addressof(table)
    assert lib2.tq_kv_append_paged_cuda(4, None, 0, None, 0, 2, 128, None, 1, None, 1, 0, None, None) == 1
    assert lib2.tq_kv_append_paged_cuda(4, None, 0, None, 0, 2, 128, C.byref(pg), 1, None, 1, 0, None, None) == 0
    pg.page_size = 48
    assert lib2.tq_kv_append_paged_cuda(4, None, 0, None, 0, 2, 128, C.byref(pg), 1, None, 1, 0, None, None) == 1
    assert pages_sizeof_matches_c()


def pages_sizeof_matches_c():
    """sizeof / offsets of tq_kv_pages in C equal the ctypes mirror."""
    import tempfile
    from leankv_b200 import attention as A
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "p.c")
        open(src, "w").write('#include "leankv_tq.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                             'int main(void){printf("%zu %zu %zu\\n", sizeof(tq_kv_pages),'
                             ' offsetof(tq_kv_pages, num_pages), offsetof(tq_kv_pages, page_size)); return 0;}\n')
        exe = os.path.join(td, "p")
        subprocess.run(["gcc", "-I", L.HEADER_DIR, src, "-o", exe], check=True)
        sz, off_n, off_p = map(int, subprocess.run([exe], capture_output=True, text=True).stdout.split())
    return sz == C.sizeof(A.KVPages) and off_n == A.KVPages.num_pages.offset and off_p == A.KVPages.page_size.offset


@pytest.mark.parametrize("args", [(0, 0, 8, 128), (65, 0, 8, 128), (2, 2, 8, 128), (2, -1, 8, 128),
                                  (2, 0, 0, 128), (2, 0, 8, 0)])
def test_peer_exchange_argument_errors(args):
    """Bad world / rank / sizes are rejected before any CUDA call (runs without a GPU)."""
    import ctypes
    lib = L.load()
    ex = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(L.TQ_PEER_HANDLE_BYTES)
    assert lib.tq_peer_exchange_create(*args, 0, ctypes.byref(ex), handle) == 1
    assert not ex.value
    assert lib.tq_peer_exchange_merge(None, None, None, 0, None, None) == 1
    assert lib.tq_peer_exchange_connect(None, None) == 1
    assert lib.tq_peer_exchange_attention(None, None, None, 0, None, None) == 1
    assert lib.tq_peer_exchange_destroy(None) == 0


def test_split_sequence_transport_name():
    from leankv_b200.distributed import SplitSequenceAttention
    with pytest.raises(ValueError, match="transport"):
        SplitSequenceAttention(transport="mpi")
