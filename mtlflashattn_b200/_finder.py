"""Import hook that serves ``flash_attn`` from this engine on CUDA hosts without flash-attn.

Contract kept from the reference's shim (_mtlflashattn_finder.py:1-96): the hook sits LAST on
``sys.meta_path``, so the regular path finders run first and an installed flash-attn always
wins; it serves exactly ``flash_attn`` and ``flash_attn.flash_attn_interface``, each exporting
the six ``flash_attn_*`` functions, ``flash_attn.__version__`` is "2.7.4" (libraries gate
features on it); ``MTLFLASHATTN_SHIM=off`` disables it; and
``importlib.metadata.packages_distributions()`` maps ``flash_attn`` to this project unless a real
distribution already claims it.

Design here: the finder answers only after a device check that runs once per process (a CUDA
device torch can see; until something imports ``flash_attn`` not even torch is imported). The
served modules are empty shells whose attributes resolve on first access through a module-level
``__getattr__`` (PEP 562), so ``import flash_attn`` stays cheap and the engine (and libmfa.so)
load only when a function is actually used.
"""
from __future__ import annotations

import functools
import importlib.abc
import importlib.machinery
import os
import sys

SERVED = ("flash_attn", "flash_attn.flash_attn_interface")
EXPORTS = (
    "flash_attn_func",
    "flash_attn_varlen_func",
    "flash_attn_qkvpacked_func",
    "flash_attn_kvpacked_func",
    "flash_attn_varlen_qkvpacked_func",
    "flash_attn_varlen_kvpacked_func",
)
DIST_NAME = "mtlflashattn-b200"


def _switched_off() -> bool:
    return os.environ.get("MTLFLASHATTN_SHIM", "auto").strip().lower() in ("off", "0", "false", "no")


@functools.lru_cache(maxsize=1)
def _cuda_present() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:  # no torch, or a broken driver: do not pretend to be flash_attn
        return False


def _lazy_exports(module):
    def __getattr__(name):
        if name in EXPORTS:
            import mtlflashattn_b200

            fn = getattr(mtlflashattn_b200, name)
            setattr(module, name, fn)  # later lookups skip this hook
            return fn
        raise AttributeError(f"module {module.__name__!r} has no attribute {name!r}")

    return __getattr__


class _ShellLoader(importlib.abc.Loader):
    """Creates the served module shells; their contents come from this engine on demand."""

    def create_module(self, spec):
        return None

    def exec_module(self, module):
        from ._version import FLASH_ATTN_SHIM_VERSION

        module.__getattr__ = _lazy_exports(module)
        module.__all__ = list(EXPORTS)
        if module.__name__ == "flash_attn":
            module.__version__ = FLASH_ATTN_SHIM_VERSION


class _MtlFlashAttnB200Finder(importlib.abc.MetaPathFinder):
    """Last-resort finder for the two served module names."""

    loader = _ShellLoader()

    def find_spec(self, fullname, path=None, target=None):
        if fullname not in SERVED or _switched_off() or not _cuda_present():
            return None
        spec = importlib.machinery.ModuleSpec(fullname, self.loader,
                                              is_package=fullname == "flash_attn")
        if fullname == "flash_attn":
            spec.submodule_search_locations = []  # a package, so the submodule resolves here
        return spec


def _claim_distribution():
    """Make ``packages_distributions()`` name this project for ``flash_attn`` when no installed
    distribution does (probes such as transformers' flash-attn availability check look it up and
    would otherwise raise KeyError on a module that imports without a distribution)."""
    import importlib.metadata as md

    current = md.packages_distributions
    if getattr(current, "__mtlflashattn_b200__", False):
        return

    @functools.wraps(current)
    def packages_distributions():
        table = current()
        table.setdefault("flash_attn", [DIST_NAME])
        return table

    packages_distributions.__mtlflashattn_b200__ = True
    md.packages_distributions = packages_distributions


def install() -> bool:
    """Append the finder to ``sys.meta_path`` once. Returns True if this call added it."""
    if _switched_off():
        return False
    if any(isinstance(f, _MtlFlashAttnB200Finder) for f in sys.meta_path):
        return False
    sys.meta_path.append(_MtlFlashAttnB200Finder())
    _claim_distribution()
    return True
