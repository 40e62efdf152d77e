"""Guarded meta-path finder that serves `flash_attn` from mtlflashattn_b200
(reference: _mtlflashattn_finder.py:1-96).

Appended to the END of sys.meta_path, so the stdlib PathFinder runs first and a real
flash_attn install always wins. Fully lazy: torch and the engine are imported only when
something imports `flash_attn`, and the finder fires only when CUDA is available.
Kill switch: MTLFLASHATTN_SHIM=off.
"""
import importlib.abc
import importlib.util
import os
import sys

_SUBMODULE_EXPORTS = (
    "flash_attn_func",
    "flash_attn_varlen_func",
    "flash_attn_qkvpacked_func",
    "flash_attn_kvpacked_func",
    "flash_attn_varlen_qkvpacked_func",
    "flash_attn_varlen_kvpacked_func",
)


def _disabled():
    return os.environ.get("MTLFLASHATTN_SHIM", "auto").lower() in ("off", "0", "false")


class _MtlFlashAttnB200Finder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    _NAMES = frozenset({"flash_attn", "flash_attn.flash_attn_interface"})

    def find_spec(self, fullname, path=None, target=None):
        if fullname not in self._NAMES or _disabled():
            return None
        try:
            import torch
            if not torch.cuda.is_available():
                return None
        except Exception:
            return None
        return importlib.util.spec_from_loader(fullname, self, is_package=(fullname == "flash_attn"))

    def create_module(self, spec):
        return None  # default module creation

    def exec_module(self, module):
        import mtlflashattn_b200 as _mfa
        from mtlflashattn_b200._version import FLASH_ATTN_SHIM_VERSION

        for name in _SUBMODULE_EXPORTS:
            setattr(module, name, getattr(_mfa, name))
        if module.__name__ == "flash_attn":
            module.__version__ = FLASH_ATTN_SHIM_VERSION


def _patch_packages_distributions():
    """Seed ``packages_distributions()["flash_attn"]`` with this project, so probes such as
    transformers' is_flash_attn_2_available() do not KeyError on a module that imports without
    a distribution, and correctly see that it is not the CUDA flash-attn distribution.
    setdefault keeps a real flash-attn install authoritative (reference: :57-83)."""
    import importlib.metadata

    orig = importlib.metadata.packages_distributions
    if getattr(orig, "_mtlflashattn_patched", False):
        return

    def packages_distributions():
        mapping = orig()
        mapping.setdefault("flash_attn", ["mtlflashattn-b200"])
        return mapping

    packages_distributions._mtlflashattn_patched = True
    importlib.metadata.packages_distributions = packages_distributions


def install():
    """Idempotently append the finder to sys.meta_path. Returns True if added."""
    if _disabled():
        return False
    if any(isinstance(f, _MtlFlashAttnB200Finder) for f in sys.meta_path):
        return False
    sys.meta_path.append(_MtlFlashAttnB200Finder())
    _patch_packages_distributions()
    return True
