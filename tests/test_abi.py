"""The C ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^[A-Za-z_][\w \t\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "while", "for", "sizeof", "return"):
                names.append(name)
    return sorted(set(names))


def test_header_declares_reference_launchers():
    names = declared_functions()
    for ref_name in ("minimax_moe_decode_topk", "moe_gemm_gguf_decode_silu"):
        assert ref_name in names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(str(pkg.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(pkg):
    assert set(declared_functions()) <= set(pkg.PROTOTYPES), set(declared_functions()) - set(pkg.PROTOTYPES)
    pkg.lib()  # binds every prototype; raises if a symbol is absent
