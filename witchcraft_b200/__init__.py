"""B200-native (sm_100a) XTR-base T5 encoder backend for dropbox/witchcraft.

The hot path is the native library libwc_t5cuda.so (CUDA kernels behind the C
ABI in include/wc_t5cuda.h).  This package holds its Python mirror of the
reference's backend interface (`t5cuda`), the build script, and the seeded
synthetic checkpoint generator (`synth`).
"""
from ._lib import WcError, lib  # noqa: F401
