"""B200 Jevstral: the Ministral-3 forward pass of theolivenbaum/llm-shield on sm_100a.

Python face of include/jv.h. The compute lives in libjv.so (CUDA, built in-tree); this
package mirrors the reference's MinistralModel / KvCache / JevstralDecider members so the
tests and the benchmark drive the same entry points a .NET host binds over P/Invoke.
"""
from ._lib import (ArgumentError, ArgumentOutOfRangeError, DeviceError, DeviceOutOfMemoryError,  # noqa: F401
                   DeviceTimeoutError, GgufIOError, InvalidDataError, JvError, NotSupportedError, NumericError,
                   OperationCanceledError, SIGNATURES, LIB_PATH)
from .decider import (DecisionResult, TokenDecider, decision_probs, margins_from_verdicts,  # noqa: F401
                      softmax)
from .layout import TokenLayout  # noqa: F401
from .model import KvCache, MinistralModel, Model, ModelConfig, Snapshot, device_count, kernel_launches  # noqa: F401
from . import dp  # noqa: F401,E402
