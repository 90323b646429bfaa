"""ctypes binding of libqwen_b200.so (declarations in include/qwen_b200.h).

The library is the product: there is no Python or CPU fallback. Importing this
module fails loudly when the in-tree shared object has not been built.
"""
import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint, c_uint16, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parents[1] / 'libqwen_b200.so'

OK, EINVAL, ETIMEOUT, EDEVICE, ETOKEN, EOUTPUT, ENOMEM, EIO, ESTATE, ESCRATCH = 0, -1, -2, -3, -4, -5, -6, -7, -8, -9
NOALLOC_SCRATCH_BYTES = 16 << 20
FLAG_RTL_KV = 1
VOCAB, HIDDEN, FFN, LAYERS = 151936, 896, 4864, 24


class Config(ctypes.Structure):
    _fields_ = [('device', c_int), ('max_seqs', c_uint32), ('max_context', c_uint32), ('max_rows', c_uint32),
                ('rms_eps', c_float), ('flags', c_uint32)]


_P8 = POINTER(ctypes.c_int8)
_P16 = POINTER(c_uint16)
_P32 = POINTER(c_uint32)
_PF = POINTER(c_float)

_SIGNATURES = {
    'qwen_b200_default_config': (None, [POINTER(Config)]),
    'qwen_b200_open': (c_int, [POINTER(Config), POINTER(c_void_p)]),
    'qwen_b200_close': (c_int, [c_void_p]),
    'qwen_b200_load_assets': (c_int, [c_void_p, c_char_p]),
    'qwen_b200_load_synthetic': (c_int, [c_void_p, c_uint64]),
    'qwen_b200_last_error': (c_char_p, [c_void_p]),
    'qwen_b200_get_config': (c_int, [c_void_p, POINTER(Config)]),
    'qwen_b200_sched_open': (c_int, [c_void_p, c_uint32, POINTER(c_void_p)]),
    'qwen_b200_sched_close': (c_int, [c_void_p]),
    'qwen_b200_sched_submit': (c_int, [c_void_p, _P32, c_uint32, c_uint32, _P32]),
    'qwen_b200_sched_step': (c_int, [c_void_p, _P32]),
    'qwen_b200_sched_result': (c_int, [c_void_p, c_uint32, _P32, c_uint32, _P32, POINTER(c_int)]),
    'qwen_b200_synth_write': (c_int, [c_char_p, c_uint64]),
    'qwen_b200_synth_prompt': (None, [c_uint64, c_uint32, _P32]),
    'qwen_b200_reset': (c_int, [c_void_p, c_uint32]),
    'qwen_b200_position': (c_int, [c_void_p, c_uint32, _P32]),
    'qwen_b200_forward': (c_int, [c_void_p, c_uint32, _P32, c_uint32, c_uint32, _P32, _P16]),
    'qwen_b200_decode_step': (c_int, [c_void_p, _P32, _P32, c_uint32, _P32]),
    'qwen_b200_prefill': (c_int, [c_void_p, c_uint32, _P32, _P32, _P32, _P32, _P16]),
    'qwen_b200_lm_head_range': (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                        c_void_p]),
    'qwen_b200_decode_step_logits': (c_int, [c_void_p, _P32, _P32, c_uint32, _P32, _P16]),
    'qwen_b200_decode_step_device': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_void_p]),
    'qwen_b200_fill_kv_synthetic': (c_int, [c_void_p, c_uint32, c_uint32, c_uint64]),
    'qwen_b200_read_kv': (c_int, [c_void_p, c_uint32, c_uint32, c_uint32, _P8, _PF, _P8, _PF]),
    'qwen_b200_read_kv_rtl': (c_int, [c_void_p, c_uint32, c_uint32, c_uint32, _P8, POINTER(ctypes.c_uint8),
                                      POINTER(ctypes.c_uint8)]),
    'qwen_b200_set_dump': (c_int, [c_void_p, c_int, _P16, _P16, _P16, _P16, _P16, _P16, _P16]),
    'qwen_b200_profile_decode': (c_int, [c_void_p, _P32, c_uint32, _P32, _PF, _P32]),
    'qwen_b200_step_launches': (c_uint32, [c_void_p]),
    'qwen_b200_csr_write': (None, [c_void_p, c_uint, c_uint64]),
    'qwen_b200_csr_read': (c_uint64, [c_void_p, c_uint]),
    'qwen_b200_embedding': (None, [c_void_p, c_uint, c_uint]),
    'qwen_b200_clear': (None, [c_void_p]),
    'qwen_b200_op_embed': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_void_p]),
    'qwen_b200_op_rmsnorm': (c_int, [c_void_p, c_void_p, c_uint32, c_float, c_void_p, c_void_p]),
    'qwen_b200_op_gemm_w8a16': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p,
                                        c_void_p, c_void_p]),
    'qwen_b200_op_gemm_w8a16_residual': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_uint32,
                                                 c_void_p, c_void_p]),
    'qwen_b200_set_persistent_decode': (c_int, [c_void_p, c_int]),
    'qwen_b200_test_expire_wait': (c_int, [c_void_p, c_int]),
    'qwen_b200_gemm_tc_workspace': (c_size_t, [c_uint32, c_uint32, c_uint32]),
    'qwen_b200_op_gemm_w8a16_tc': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p,
                                           c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    'qwen_b200_rope_table': (None, [c_uint32, _PF]),
    'qwen_b200_op_rope': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    'qwen_b200_op_kv8_append': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                        c_void_p]),
    'qwen_b200_op_k16_append': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_uint32, c_void_p]),
    'qwen_b200_op_v8_append': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_uint32, c_void_p]),
    'qwen_b200_op_qkv': (c_int, [c_void_p, c_uint32, c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                 c_void_p]),
    'qwen_b200_attention_workspace': (c_size_t, [c_uint32, c_uint32]),
    'qwen_b200_op_attention': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_uint32, c_void_p, c_void_p, c_size_t, c_void_p]),
    'qwen_b200_op_attention_noalloc': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p,
                                               c_void_p, c_void_p, c_void_p, c_uint32, c_void_p, c_void_p]),
    'qwen_b200_op_attention_cluster': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p,
                                               c_void_p, c_void_p, c_void_p, c_uint32, c_void_p, c_void_p]),
    'qwen_b200_attention_prefill_workspace': (c_size_t, [c_uint32]),
    'qwen_b200_op_attention_prefill': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p,
                                               c_uint32, c_void_p, c_void_p, c_size_t, c_void_p]),
    'qwen_b200_op_swiglu': (c_int, [c_void_p, c_uint32, c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    'qwen_b200_lm_head_workspace': (c_size_t, [c_uint32, c_uint32]),
    'qwen_b200_op_lm_head_argmax': (c_int, [c_void_p, c_uint32, c_void_p, c_float, c_void_p, c_void_p, c_uint32,
                                            c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib = None


def lib():
    """Loads the in-tree libqwen_b200.so once and declares every entry point."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f'{LIB_PATH} is not built; run `python -m qwen_b200.build` '
                               '(there is no fallback implementation)')
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class QwenError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f'libqwen_b200 status {status}: {message}')
        self.status = status


def check(status, handle=None):
    if status != OK:
        msg = lib().qwen_b200_last_error(handle).decode(errors='replace') if handle else ''
        raise QwenError(status, msg)
    return status


def u32(values):
    arr = (c_uint32 * len(values))(*values)
    return arr


def ptr(array, ctype):
    """Pointer to a numpy array's data."""
    return array.ctypes.data_as(POINTER(ctype))
