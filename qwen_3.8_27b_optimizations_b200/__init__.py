"""B200-native (sm_100a) IQ4_XS x Q8_1 quantised matmul: the reference's hot path rebuilt.

The directory name contains dots, so it is loaded by path (see tests/conftest.py,
__graft_entry__.py, bench.py) under the module name ``iq4xs_b200``.
"""
from .api import *  # noqa: F401,F403
from .api import lib, LIB_PATH, SIGNATURES, IQ4XSError  # noqa: F401
from . import peer  # noqa: F401,E402  (collectives over NVLink peer memory)
from . import sharded  # noqa: F401,E402  (row-sharded multi-GPU matmuls)
from . import decoder  # noqa: F401,E402  (synthetic tensor-parallel decoder)
from . import gguf_weights  # noqa: F401,E402  (IQ4_XS matrices from / to GGUF files)
