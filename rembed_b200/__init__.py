"""rembed_b200: a B200-native (sm_100a) encoder forward pass for rembed.

The product is ``librembed_gpu.so`` (C ABI declared in
``include/rembed_gpu.h``): hand-written CUDA kernels behind the
init / upload-weights / forward / free interface that rembed's Go host
calls in place of its pure-Go ``internal/tensor`` kernels.  This Python
package is the host-side mirror of the reference's public API
(``rembed.Load`` / ``Embed`` / ``EmbedTokens`` / ``WithInt8`` /
``WithInt8Activations`` / ``WithDim``) over that ABI, for Python callers
and for the parity tests.
"""

from .config import Config, ConfigError  # noqa: F401
from .embedder import Embedder, RembedError, load  # noqa: F401
