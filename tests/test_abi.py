"""CPU: the C-ABI library loads and exports every symbol include/*.h declares.

No compute calls (this container has no GPU)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER_DIR = ROOT / "include"


def declared_functions():
    names = []
    for h in HEADER_DIR.glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        # function declarations (callback typedefs are types, not symbols)
        for m in re.finditer(r"^\s*(?!typedef\b)(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([a-z_][a-z0-9_]*)\s*\(", text,
                             flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_reference_entry_points():
    names = declared_functions()
    # the reference's C ABI for this path (python/gpu_eigsh/_bindings.cpp:19-30)
    assert "compute_eigsh" in names and "compute_eigsh_sigma" in names
    assert "lg_eigsh_plan_create" in names and "lg_eigsh_plan_run" in names
    # matrix-free operators (src/matvec_operator.cuh:149-163 FunctionOperator)
    assert "lg_eigsh_plan_create_op" in names


def test_library_exports_every_declared_symbol():
    from gpu_eigsh import _native

    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"symbols declared in include/*.h but not exported: {missing}"
    # and the Python binding knows a signature for each of them
    unbound = [n for n in declared_functions() if n not in _native.SIGNATURES]
    assert not unbound, f"no ctypes signature for: {unbound}"


def test_library_is_sm100a_only_build():
    # the shared object was produced by nvcc for sm_100a; its presence and the
    # build recipe are what the product path relies on (no CPU fallback)
    from gpu_eigsh import _native

    assert Path(_native.LIB_PATH).name == "liblanczos_b200.so"
    build_py = (ROOT / "lanczos-gpu_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in build_py


def test_status_strings_without_gpu():
    from gpu_eigsh import _native

    assert _native.status_string(0) == "ok"
    assert "CG" in _native.status_string(_native.LG_ERR_CG_NOCONV)


def test_info_record_matches_header():
    """The ctypes view of lg_eigsh_info has one slot per kernel class of the
    header's enum (LG_K_SPMV ... LG_K_COMM, LG_K_CLASSES), in the same order,
    so the per-class device times land under the right names."""
    from gpu_eigsh import _native

    text = (HEADER_DIR / "lanczos_b200.h").read_text()
    enum = {m.group(1): int(m.group(2)) for m in re.finditer(r"\b(LG_K_[A-Z_]+)\s*=\s*(\d+)", text)}
    n = enum.pop("LG_K_CLASSES")
    assert n == len(_native.KERNEL_CLASSES)
    assert sorted(enum.values()) == list(range(n))
    names = {"LG_K_SPMV": "spmv", "LG_K_PROJECT": "gs_project", "LG_K_CORRPROJ": "gs_correct_project",
             "LG_K_CORRECT": "gs_correct", "LG_K_RESTART": "restart", "LG_K_BASIS": "basis", "LG_K_CG": "cg",
             "LG_K_OTHER": "other", "LG_K_COMM": "comm"}
    for k, v in enum.items():
        assert _native.KERNEL_CLASSES[v] == names[k]
    # the arrays are sized by LG_K_CLASSES in the header
    assert "kernel_ms[LG_K_CLASSES]" in text
    fields = dict(_native.EigshInfo._fields_)
    assert fields["kernel_ms"]._length_ == n and fields["kernel_calls"]._length_ == n
