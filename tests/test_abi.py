"""C-ABI library: loads and exports every symbol the header declares (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "yapd_select.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(yapd_\w+)\s*\(", txt, re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "yapd_select_step" in syms and "yapd_sample_rows" in syms


def test_library_exports_all_declared_symbols():
    from yapd_b200.build import build
    lib_path = build()
    lib = ctypes.CDLL(lib_path)
    for s in declared_symbols():
        assert hasattr(lib, s), f"missing export {s}"


def test_binding_matches_header():
    from yapd_b200 import _native as N
    assert set(N.EXPORTED) == set(declared_symbols())
    lib = N.lib()
    assert lib.yapd_abi_version() == N.YAPD_ABI_VERSION
    hdr = open(os.path.join(ROOT, "include", "yapd_select.h")).read()
    assert re.search(r"#define YAPD_ABI_VERSION %d\b" % N.YAPD_ABI_VERSION, hdr)
    assert lib.yapd_select_workspace_size(64, 32) >= 64 * 32 * 4
    assert b"NULL" in lib.yapd_status_string(-1)


def test_host_validation_without_gpu():
    """Invalid arguments are rejected on the host before any CUDA call."""
    import ctypes as C
    from yapd_b200 import _native as N
    lib = N.lib()
    a = N.SelectArgs()
    assert lib.yapd_select_step(C.byref(a), None) == -2          # B = 0
    a.B, a.nb, a.L, a.V, a.K = 1, 2, 16, 9000, 4
    assert lib.yapd_select_step(C.byref(a), None) == -5          # V too large
    a.V = 8194
    a.logits_dtype = 7
    assert lib.yapd_select_step(C.byref(a), None) == -3
    a.logits_dtype = 1
    assert lib.yapd_select_step(C.byref(a), None) == -1          # NULL pointers
    a.L = 33
    assert lib.yapd_select_step(C.byref(a), None) == -2          # L > 32
    assert lib.yapd_sample_rows(None, None) == -1


def test_history_stride_checked():
    """A history row shorter than the vocabulary is rejected (no out-of-row reads)."""
    import ctypes as C
    from yapd_b200 import _native as N
    lib = N.lib()
    a = N.SampleArgs()
    a.R, a.V, a.logits_dtype = 4, 8194, N.YAPD_DTYPE_F32
    a.logits, a.sampled = 4096, 4096            # never dereferenced: rejected on the host
    a.stride_row, a.logits_numel = 8194, 4 * 8194
    a.workspace, a.workspace_bytes = 4096, 256
    a.sampling.history_kind = N.YAPD_HISTORY_BITMAP
    a.sampling.history = 4096
    a.sampling.history_stride = (8194 + 31) // 32 - 1
    assert lib.yapd_sample_rows(C.byref(a), None) == -2
    a.sampling.history_kind = N.YAPD_HISTORY_BYTES
    a.sampling.history_stride = 8193
    assert lib.yapd_sample_rows(C.byref(a), None) == -2


def test_noalloc_checks_before_enqueue():
    """yapd_select_step_noalloc rejects bad arguments before touching the stream
    (an invalid stream handle is never used)."""
    import ctypes as C
    from yapd_b200 import _native as N
    lib = N.lib()
    a = N.SelectArgs()
    a.B, a.nb, a.L, a.V, a.K = 2, 2, 16, 8194, 4
    a.logits_dtype = 5
    assert lib.yapd_select_step_noalloc(C.byref(a), C.c_void_p(0xdead)) == -3


def test_ctypes_layout_matches_c():
    """The ctypes mirror of the argument structs has the C compiler's layout
    (sizes and the offset of every field), checked with the host gcc."""
    import ctypes as C
    import shutil
    import subprocess
    import tempfile
    from yapd_b200 import _native as N
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    structs = {"yapd_sampling": N.Sampling, "yapd_noise": N.Noise, "yapd_engine_state": N.EngineState,
               "yapd_select_args": N.SelectArgs, "yapd_sample_args": N.SampleArgs,
               "yapd_lmhead_args": N.LmheadArgs}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "yapd_select.h"', "int main(void) {"]
    want = []
    for cname, py in structs.items():
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        want.append(C.sizeof(py))
        for fname, _ in py._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {fname}));')
            want.append(getattr(py, fname).offset)
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(src, "w").write("\n".join(lines))
        subprocess.run([cc, "-I", os.path.join(ROOT, "include"), "-o", exe, src], check=True)
        got = [int(x) for x in subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()]
    assert got == want


def test_lmhead_validation_without_gpu():
    """The fused head's host checks: shapes, alignment and the sampling chain
    it serves are rejected before any CUDA call."""
    import ctypes as C
    from yapd_b200 import _native as N
    lib = N.lib()
    h = N.LmheadArgs()
    assert lib.yapd_lmhead_select_step(None, None) == -1
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -2      # B = 0
    a = h.select
    a.B, a.nb, a.L, a.V, a.K = 4, 2, 32, 8194, 8
    h.D = 1000
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -2      # D not a multiple of 64
    h.D = 1024
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -1      # NULL hidden / weight
    h.hidden, h.weight = 4096 + 8, 4096
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -4      # hidden not 16-byte aligned
    h.hidden = 4096
    h.h_stride_req, h.h_stride_branch, h.h_stride_pos = 2 * 32 * 1024, 32 * 1024, 1024
    h.hidden_numel, h.w_stride, h.weight_numel = 4 * 2 * 32 * 1024, 1024, 8194 * 1024
    for f in ("xt", "k_step", "is_commit", "log_prior", "sched_t", "q_t", "xt_out", "sampled", "pmi",
              "n_unmask", "n_mask_after", "hit_eos", "k_step_out", "is_commit_out", "workspace"):
        setattr(a, f, 4096)
    a.workspace_bytes = lib.yapd_lmhead_workspace_size(4, 32)
    a.sampling.top_p_s = 0.9
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -8      # top-p is not on this path
    a.sampling.top_p_s = 1.0
    a.sampling.min_p_s = 0.05
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -8      # nor min-p
    a.sampling.min_p_s = 0.0
    a.nb = 1
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -2      # CFG rows only
    a.nb, a.L = 2, 24
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -2      # L of 16 or 32
    a.L = 32
    a.workspace_bytes = 256
    assert lib.yapd_lmhead_select_step(C.byref(h), None) == -6      # workspace too small
