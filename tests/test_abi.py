"""The C-ABI library loads and exports every entry point include/g4q.h declares (no GPU needed)."""
import ctypes
import re

import pytest

from conftest import ROOT


def declared_functions():
    text = (ROOT / "include" / "g4q.h").read_text()
    return sorted(set(re.findall(r"^G4qStatus\s+(g4q_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("g4q_weight_create", "g4q_weight_load", "g4q_qmm", "g4q_dequantize", "g4q_lm_head_argmax",
                     "g4q_get_last_error", "g4q_runtime_version"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from helios_b200 import _lib
    L = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding declares a signature for every exported entry point
    assert set(declared_functions()) <= set(_lib.SIGNATURES), set(declared_functions()) - set(_lib.SIGNATURES)


def test_version_and_last_error_without_gpu():
    from helios_b200 import _lib
    v = _lib.version()
    assert v["abi_version"] == 1 and v["backend_name"] == "g4q_b200"
    assert _lib.last_error() == ""


def test_status_and_message_on_invalid_arguments_without_gpu():
    from helios_b200 import _lib
    L = _lib.load()
    st = L.g4q_weight_create(64, 128, 4, 64, None)
    assert st == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "non-null out pointer" in _lib.last_error()
    st = L.g4q_qmm(None, None, 1, 64, None, 64, None)
    assert st == _lib.G4Q_ERR_INVALID_ARGUMENT
    assert "weight handle" in _lib.last_error()
    bogus = ctypes.create_string_buffer(256)       # not a handle: the magic check rejects it
    st = L.g4q_weight_free(ctypes.cast(bogus, ctypes.c_void_p))
    assert st == _lib.G4Q_ERR_INVALID_ARGUMENT and "invalid weight handle" in _lib.last_error()
    assert L.g4q_get_last_error(None, 0) == _lib.G4Q_ERR_INVALID_ARGUMENT
    with pytest.raises(_lib.G4qInvalidArgument):
        _lib.call("g4q_runtime_version", None)


def test_plan_comm_ipc_and_noalloc_reject_bad_arguments_without_gpu():
    """Handles, ranks, sizes and pointers are checked on the host before any CUDA call, so every one
    of these returns G4Q_ERR_INVALID_ARGUMENT with its message on a machine without a GPU."""
    from helios_b200 import _lib
    L = _lib.load()
    bogus = ctypes.cast(ctypes.create_string_buffer(256), ctypes.c_void_p)
    p = ctypes.c_void_p(256)                        # never dereferenced: validation fails first
    out, words, nbytes = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_uint64()
    cases = [
        (lambda: L.g4q_decode_plan_run(None, 1, 1e-6, 30.0, 0, None, None, None, None, 0, None),
         "invalid decode plan handle"),
        (lambda: L.g4q_decode_plan_run(bogus, 1, 1e-6, 30.0, -1, None, None, None, None, 0, None),
         "row_offset out of range"),
        (lambda: L.g4q_decode_plan_free(bogus), "invalid decode plan handle"),
        (lambda: L.g4q_decode_plan_trace(bogus, None, None), "words must be non-null"),
        (lambda: L.g4q_decode_plan_trace(bogus, None, ctypes.byref(words)), "invalid decode plan handle"),
        (lambda: L.g4q_decode_plan_buffers(bogus, ctypes.byref(out), ctypes.byref(nbytes), ctypes.byref(out),
                                           ctypes.byref(nbytes)), "invalid decode plan handle"),
        (lambda: L.g4q_decode_plan_create(None, 1, 1, None), "non-null out pointer"),
        (lambda: L.g4q_decode_plan_create_ex(None, None, 0, 1, 0, 1, ctypes.byref(out)), "at least one phase"),
        (lambda: L.g4q_comm_create(0, 2, 16, None), "non-null out pointer"),
        (lambda: L.g4q_comm_create(2, 2, 16, ctypes.byref(out)), "rank must be in [0, n_ranks)"),
        (lambda: L.g4q_comm_create(0, 9, 16, ctypes.byref(out)), "1 <= n_ranks <= 8"),
        (lambda: L.g4q_comm_create(0, 2, 0, ctypes.byref(out)), "max_elems must be in [1, 2^31]"),
        (lambda: L.g4q_comm_free(bogus), "invalid communicator handle"),
        (lambda: L.g4q_allreduce(bogus, p, 8, 0, None), "invalid communicator handle"),
        (lambda: L.g4q_ipc_handle(None, None), "non-null pointers"),
        (lambda: L.g4q_ipc_open(None, None), "non-null pointers"),
        (lambda: L.g4q_ipc_close(None), "non-null pointer"),
        (lambda: L.g4q_device_error(None, 0), "non-null code pointer"),
        (lambda: L.g4q_lm_head_argmax_noalloc(None, None, 16, 64, None, 1, 64, 30.0, 0, 1e-6, 0, None, 0,
                                              None, None, None, None), "non-null device pointers"),
        (lambda: L.g4q_lm_head_argmax_noalloc(p, p, 16, 64, p, 17, 64, 30.0, 0, 1e-6, 0, None, 0,
                                              None, None, None, None), "M must be in [1, 16]"),
        (lambda: L.g4q_lm_head_argmax_noalloc(p, p, 15, 64, p, 1, 64, 30.0, 0, 1e-6, 0, None, 0,
                                              None, None, None, None), "positive multiple of 16"),
        (lambda: L.g4q_dequantize_mlx(None, None, None, 16, 64, 4, 64, 0, None, None), "non-null"),
    ]
    for call, message in cases:
        assert call() == _lib.G4Q_ERR_INVALID_ARGUMENT, message
        assert message in _lib.last_error(), (message, _lib.last_error())


def test_missing_library_fails_loudly(tmp_path):
    from helios_b200 import _lib
    saved = _lib._lib
    try:
        _lib._lib = None
        with pytest.raises(_lib.G4qUnavailable):
            _lib.load(tmp_path / "nope.so")
    finally:
        _lib._lib = saved


# Public structs whose layout the bindings (ctypes here, a Rust #[repr(C)] mirror for the reference's
# host) depend on: name -> fields, in declaration order.
PINNED = {
    "G4qVersionInfo": ["abi_version", "backend_name", "backend_version"],
    "G4qWeightInfo": ["rows", "cols", "bits", "group_size", "device_bytes", "device", "fast_path_ok", "error_flags"],
    "G4qDecodePhase": ["weight", "x", "ldx", "y", "ldy", "flags"],
    "G4qPhasePrologue": ["post_norm_weight", "residual", "layer_scalar", "norm_weight", "residual_out",
                         "ld_residual_out", "eps"],
}


def test_struct_layouts_match_the_binding(tmp_path):
    """Layout pins of the C ABI's structs: sizeof / offsetof from the C compiler on include/g4q.h
    equal the ctypes binding's, field by field (a binding built from the header cannot drift)."""
    import shutil
    import subprocess

    from helios_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include "g4q.h"', "#include <stddef.h>", "#include <stdio.h>", "int main(void) {"]
    for s, fields in PINNED.items():
        lines.append(f'    printf("{s} size %zu\\n", sizeof({s}));')
        for f in fields:
            lines.append(f'    printf("{s} {f} %zu\\n", offsetof({s}, {f}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "pins.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "pins"
    subprocess.run([cc, "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        s, f, v = ln.split()
        got[(s, f)] = int(v)
    for s, fields in PINNED.items():
        cls = getattr(_lib, s)
        assert [f for f, _ in cls._fields_] == fields, s
        assert got[(s, "size")] == ctypes.sizeof(cls), s
        for f in fields:
            assert got[(s, f)] == getattr(cls, f).offset, (s, f)


C_HOST = r'''
#include "g4q.h"
#include <pthread.h>
#include <stdio.h>
#include <string.h>

static int expect(G4qStatus got, G4qStatus want, const char* needle) {
    char msg[512];
    if (got != want) { printf("status %d, expected %d\n", (int)got, (int)want); return 1; }
    if (g4q_get_last_error(msg, sizeof msg) != G4Q_OK) return 1;
    if (needle && !strstr(msg, needle)) { printf("message '%s' lacks '%s'\n", msg, needle); return 1; }
    if (!needle && msg[0]) { printf("message '%s' after success\n", msg); return 1; }
    return 0;
}

static void* other_thread(void* arg) {
    char msg[512];
    int* bad = (int*)arg;
    g4q_get_last_error(msg, sizeof msg);
    if (msg[0]) { printf("thread sees '%s'\n", msg); *bad = 1; }
    *bad |= expect(g4q_decode_plan_free(NULL), G4Q_ERR_INVALID_ARGUMENT, "invalid decode plan handle");
    return NULL;
}

int main(void) {
    G4qVersionInfo v;
    G4qWeight* w = NULL;
    pthread_t t;
    char small[8];
    int bad = 0;
    bad |= expect(g4q_runtime_version(&v), G4Q_OK, NULL);
    if (v.abi_version != G4Q_ABI_VERSION || strcmp(v.backend_name, "g4q_b200") != 0) bad = 1;
    bad |= expect(g4q_weight_create(64, 128, 4, 64, NULL), G4Q_ERR_INVALID_ARGUMENT, "non-null out pointer");
    bad |= expect(g4q_weight_create(64, 128, 3, 64, &w), G4Q_ERR_UNSUPPORTED_CONFIG, "bits=3");
    bad |= expect(g4q_weight_create(60, 128, 4, 64, &w), G4Q_ERR_UNSUPPORTED_CONFIG, "multiple of 16");
    if (w != NULL) bad = 1;
    /* the last error is per thread: another thread neither sees nor overwrites this one */
    if (pthread_create(&t, NULL, other_thread, &bad) != 0 || pthread_join(t, NULL) != 0) return 3;
    bad |= expect(G4Q_ERR_UNSUPPORTED_CONFIG, G4Q_ERR_UNSUPPORTED_CONFIG, "multiple of 16");
    /* a short buffer receives a terminated prefix */
    if (g4q_get_last_error(small, sizeof small) != G4Q_OK || strlen(small) != sizeof small - 1) bad = 1;
    if (g4q_get_last_error(NULL, 0) != G4Q_ERR_INVALID_ARGUMENT) bad = 1;
    /* a successful call clears it */
    bad |= expect(g4q_runtime_version(&v), G4Q_OK, NULL);
    printf("%s %s: %s\n", v.backend_name, v.backend_version, bad ? "FAIL" : "ok");
    return bad;
}
'''


def test_c_host_program_links_and_reads_statuses(tmp_path):
    """A C host (as the reference's Rust crate or C++ runtime would be) compiled against the header
    with strict warnings, linked to the library: version, statuses and the per-thread last error,
    all of which work without a GPU."""
    import shutil
    import subprocess
    from pathlib import Path

    from helios_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    so = Path(_lib.load()._name)
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(src),
                    "-o", str(exe), "-L", str(so.parent), "-lg4q", f"-Wl,-rpath,{so.parent}", "-pthread"],
                   check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith(": ok"), r.stdout
