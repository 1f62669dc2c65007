"""TriFusion-FP fused Mamba-3 recurrence for NVIDIA B200 (sm_100a).

Drop-in for the reference package ``trifusion_l4`` (``__init__.py:10-35``):
the same public names load lazily, so importing the package pulls in neither
torch nor the CUDA library.
"""

from importlib import import_module

__version__ = "0.1.0"
__all__ = ["__version__", "configure_runtime", "load_student", "InferenceEngine", "fused_mamba"]

_EXPORTS = {
    "configure_runtime": (".runtime", "configure_runtime"),
    "load_student": (".runtime", "load_student"),
    "InferenceEngine": (".runtime", "InferenceEngine"),
    "fused_mamba": (".mamba_fused", "fused_mamba"),
    "fused_recurrence": (".mamba_fused", "fused_recurrence"),
    "check_device_error": ("._lib", "check_device_error"),
}


def __getattr__(name):
    if name not in _EXPORTS:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    module_name, attribute = _EXPORTS[name]
    value = getattr(import_module(module_name, __name__), attribute)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(__all__))
