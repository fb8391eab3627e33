"""Access to the reference's own operator programs for the plugin tests.

The arrangement/application pairs live in the reference's tests/test_*.py.
They are loaded from the reference installed in baseline/_ref (the unmodified
`ninetoothed` package plus the reference test modules in
baseline/_ref/reference_tests), or from NINETOOTHED_REFERENCE (a source tree
with src/ and tests/).  The reference test modules import each other as
`tests.<name>`; they are registered under those names while loaded.
"""

import importlib.util
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _locate():
    installed = REPO / "baseline" / "_ref"
    if (installed / "ninetoothed").is_dir() and (installed / "reference_tests").is_dir():
        return installed, installed / "reference_tests"
    tree = os.environ.get("NINETOOTHED_REFERENCE")
    if tree and (Path(tree) / "src" / "ninetoothed").is_dir():
        return Path(tree) / "src", Path(tree) / "tests"
    return None, None


PACKAGE_DIR, TESTS_DIR = _locate()
AVAILABLE = PACKAGE_DIR is not None


def import_ninetoothed():
    if str(PACKAGE_DIR) not in sys.path:
        sys.path.insert(0, str(PACKAGE_DIR))
    import ninetoothed

    return ninetoothed


def load(name):
    """The reference test module `name` (e.g. "test_matmul")."""
    import_ninetoothed()
    key = f"tests.{name}"
    module = sys.modules.get(key)
    if module is not None and getattr(module, "__file__", "").startswith(str(TESTS_DIR)):
        return module
    for dependency in ("utils", "test_matmul"):
        dep_key = f"tests.{dependency}"
        if dependency != name and dep_key not in sys.modules:
            _exec(dependency)
    return _exec(name)


def _exec(name):
    spec = importlib.util.spec_from_file_location(f"tests.{name}", TESTS_DIR / f"{name}.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules[f"tests.{name}"] = module
    spec.loader.exec_module(module)
    return module
