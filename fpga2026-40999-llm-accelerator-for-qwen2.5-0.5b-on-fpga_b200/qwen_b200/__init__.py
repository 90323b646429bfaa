"""Host side of libqwen_b200: ctypes binding of the C ABI (include/qwen_b200.h),
an in-tree build script, and `Model`, the mirror of the reference's
behavioural-model interface (legacy_100mhz_closed/src/PC/model_backend.py)."""
from ._lib import FLAG_RTL_KV, LIB_PATH, QwenError, lib  # noqa: F401
from .model import Engine, Model, Scheduler, bf16_to_f32  # noqa: F401
