"""Loader of the in-tree native binding.  There is no fallback: if the shared objects are
missing the import fails loudly with the build command to run."""
from __future__ import annotations

import importlib.machinery
import importlib.util
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIBRARY = _PKG / "libtrring.so"
BINDING = _PKG / "_trring_torch.so"
_module = None


def binding():
    """The compiled torch binding (_trring_torch), loaded from the package directory."""
    global _module
    if _module is None:
        if not BINDING.exists() or not LIBRARY.exists():
            raise RuntimeError(
                f"kernel_task_b200 native code is not built ({BINDING.name}, {LIBRARY.name} "
                f"missing in {_PKG}); run `python -m kernel_task_b200.build`")
        import torch  # noqa: F401  (libtorch must be loaded before the binding)

        loader = importlib.machinery.ExtensionFileLoader("_trring_torch", str(BINDING))
        spec = importlib.util.spec_from_file_location("_trring_torch", str(BINDING),
                                                      loader=loader)
        module = importlib.util.module_from_spec(spec)
        loader.exec_module(module)
        _module = module
    return _module
