"""omni-tokenizer hot path for NVIDIA B200 (sm_100a).

The directory name (omni-tokenizer_b200) is not a Python identifier; import it
as `omni_tokenizer_b200` through load_package() in tests/conftest.py,
bench.py or __graft_entry__.py, or bind libomni_b200.so directly with ctypes
(native.py declares every op-level signature, abi.py the omni_* ones).
"""

from .native import NativeError, Library, Context, library, attention_bhld, attention_rows, gelu_  # noqa: F401

__version__ = "0.1.0"
