"""CPU tests of the C-ABI boundary: the library builds for sm_100a, loads
without a GPU, exports every symbol include/rta.h declares, rejects bad
arguments with a status code (host-side validation, no device work), and its
Python mirror (ctypes signatures, the model-spec struct) matches the header."""
import ctypes
import re
import shutil
import subprocess

import pytest

from rta_b200 import _build, _lib


def test_library_builds_and_exports_header_symbols():
    lib = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib._SIGNATURES) <= set(names)
    assert lib.rta_version().decode().endswith("sm_100a")


def test_argument_validation_without_device():
    lib = _lib.load()
    assert lib.rta_gemv(12, None, 16, 256, None, 1, None, 0, None) == _lib.RTA_E_ARG
    assert b"rta_gemv" in lib.rta_last_error()
    assert lib.rta_quantize(3, None, 1, None, None) == _lib.RTA_E_ARG
    assert lib.rta_readout(14, None, 16, 256, None, 9, None, None, None, None, None) == _lib.RTA_E_ARG
    word = ctypes.c_uint32(0)
    assert lib.rta_workspace_error(None, 0, None, ctypes.byref(word)) == _lib.RTA_E_ARG
    assert lib.rta_attention_workspace_bytes(16, 4, 256, 8) > 16 * 8 * 256 * 4



_SCALARS = {"int": ctypes.c_int, "rta_status": ctypes.c_int, "uint32_t": ctypes.c_uint32,
            "uint64_t": ctypes.c_uint64, "size_t": ctypes.c_size_t, "float": ctypes.c_float,
            "double": ctypes.c_double}


def _header_declarations():
    """name -> (return type, [parameter types]) for every RTA_API function of
    include/*.h; a parameter or return with '*' or '[' reads as "pointer"."""
    def kind(decl):
        decl = decl.strip()
        if "*" in decl or "[" in decl:
            return "pointer"
        words = [w for w in decl.split() if w != "const"]
        return words[0] if len(words) == 1 else " ".join(words[:-1])

    out = {}
    for h in sorted(_build.INCLUDE.glob("*.h")):
        for ret, name, params in re.findall(r"^RTA_API\s+([\w\s\*]+?)\s*\b(rta_\w+)\s*\(([^)]*)\)\s*;",
                                             h.read_text(), flags=re.M):
            plist = [p for p in (x.strip() for x in params.split(",")) if p and p != "void"]
            out[name] = ("pointer" if "*" in ret else ret.replace("const", "").strip(), [kind(p) for p in plist])
    return out


def _is_pointer(t):
    return t in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(t, type) and issubclass(t, ctypes._Pointer))


def test_bindings_match_header_declarations():
    """Every ctypes binding (operators and the model handle) has the arity and
    the scalar / pointer kind of each argument and of the result that the
    header declares, so the Python mirror cannot drift from the C-ABI."""
    from rta_b200 import model
    decls = _header_declarations()
    assert set(decls) == set(_lib.header_symbols())
    bindings = dict(_lib._SIGNATURES)
    bindings.update(model._SIGS)
    assert set(bindings) <= set(decls), sorted(set(bindings) - set(decls))
    for name, (res, args) in bindings.items():
        ret, params = decls[name]
        assert len(args) == len(params), (name, len(args), len(params))
        for i, (have, want) in enumerate(zip(args, params)):
            if want == "pointer":
                assert _is_pointer(have), (name, i, have)
            else:
                assert have is _SCALARS[want], (name, i, have, want)
        if ret == "void":
            assert res is None, name
        elif ret == "pointer":
            assert _is_pointer(res), (name, res)
        else:
            assert res is _SCALARS[ret], (name, res, ret)


def test_model_spec_mirror_has_the_c_layout(tmp_path):
    """The ctypes mirror of rta_model_spec has the size and field offsets that a
    C compiler gives the header's struct (the handle reads it by value)."""
    from rta_b200.model import ModelSpecC
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in ModelSpecC._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"rta.h\"\nint main(void) {\n"
                   "  printf(\"%zu\\n\", sizeof(rta_model_spec));\n"
                   + "".join(f"  printf(\"%zu\\n\", offsetof(rta_model_spec, {f}));\n" for f in fields)
                   + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(_build.INCLUDE), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert got[0] == ctypes.sizeof(ModelSpecC)
    assert got[1:] == [getattr(ModelSpecC, f).offset for f in fields]
