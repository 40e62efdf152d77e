"""Explicit opt-in registration of the guarded `flash_attn` shim
(reference: metal_flash_attn/_shim.py:9-12).

Installs add ``mtlflashattn_b200_autoload.pth`` to site-packages to register it at interpreter
start; call install() where that mechanism is unavailable (embedded interpreters, zipapps).
"""


def install():
    from . import _finder

    return _finder.install()
