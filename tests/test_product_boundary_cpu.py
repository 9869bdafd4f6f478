"""The product package never reaches the oracle and has no CPU fallback:
no module of cxlsparse_b200 imports oracle/ (nor a tracing compiler), and a
missing shared library is an ImportError, not a silent slow path."""

import ast
from pathlib import Path

import pytest

from cxlsparse_b200 import _lib

PACKAGE = Path(_lib.__file__).resolve().parent


def _imports(path):
    tree = ast.parse(path.read_text(), str(path))
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            yield from (alias.name for alias in node.names)
        elif isinstance(node, ast.ImportFrom) and node.level == 0 and node.module:
            yield node.module


@pytest.mark.parametrize("path", sorted(PACKAGE.glob("*.py")), ids=lambda p: p.name)
def test_package_imports_neither_oracle_nor_a_tracing_compiler(path):
    for name in _imports(path):
        root = name.split(".")[0]
        assert root not in ("oracle", "triton", "tilelang"), (path.name, name)
    assert "torch.compile" not in path.read_text(), path.name


def test_missing_library_raises_instead_of_falling_back(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "libcxlsparse_b200.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError, match="no CPU fallback"):
        _lib.lib()
