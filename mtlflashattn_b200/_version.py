__version__ = "0.1.0"

# Version the guarded `flash_attn` shim reports. Libraries feature-gate on
# flash_attn.__version__ (e.g. ">=2.3" for window_size), so it must parse as a flash-attn 2.x
# release; same value as the reference (metal_flash_attn/_version.py:6).
FLASH_ATTN_SHIM_VERSION = "2.7.4"
