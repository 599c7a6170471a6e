"""sigcomp_b200: B200-native neural codec for SigComp's compression hot path.

The package replaces the device half of SigComp's codec object
(``GPUCompression``, built by ``_load_model`` in sigcomp/main.py:189-225) with
hand-written sm_100a CUDA kernels behind the C ABI in include/sigcomp_b200.h.
"""

from .model import IntModel, load_model, random_model  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # the codec loads the CUDA library; import it lazily so CPU-only users of
    # the host helpers (model loading, signal transform) never touch it
    if name in ("B200Compression", "GPUCompression"):
        from . import codec
        return getattr(codec, name)
    raise AttributeError(name)
