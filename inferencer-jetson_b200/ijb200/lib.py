"""ctypes binding of include/ijb200.h."""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# IJB200_LIB selects another build of the same library (e.g. to compare two builds on one GPU)
LIB_PATH = os.environ.get("IJB200_LIB") or os.path.join(PKG_ROOT, "lib", "libijb200.so")
REPO_ROOT = os.path.dirname(PKG_ROOT)
HEADER = os.path.join(REPO_ROOT, "include", "ijb200.h")

OK = 0
ERR_INVALID, ERR_CUDA, ERR_NOMEM, ERR_CAPACITY, ERR_DEVICE = 1, 2, 3, 4, 5
GEMV_PDL = 2  # IJB_GEMV_PDL: ijb_gemv flag bit

_lib = None


class IjbError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[ijb error {code}] {msg}")
        self.code = code


class ModelDesc(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("hidden", ctypes.c_int), ("vocab", ctypes.c_int),
                ("eps", ctypes.c_float), ("rope_base", ctypes.c_float), ("context", ctypes.c_int),
                ("max_batch", ctypes.c_int), ("max_seqs", ctypes.c_int), ("page_size", ctypes.c_int),
                ("num_pages", ctypes.c_long), ("use_dp4a", ctypes.c_int), ("use_q6_dp4a", ctypes.c_int),
                ("kv_f32", ctypes.c_int), ("device", ctypes.c_int)]


class TensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int), ("n_dims", ctypes.c_int),
                ("dims", ctypes.c_int64 * 4), ("data_dev", ctypes.c_void_p)]


def build() -> str:
    """Compile libijb200.so for sm_100a with the package Makefile."""
    subprocess.run(["make", "-s", "-C", PKG_ROOT], check=True)
    return LIB_PATH


def load():
    """Load libijb200.so (fails loudly when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
                           "(there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, L64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
    IP = ctypes.POINTER(ctypes.c_int)
    sig = {
        "ijb_create": ([ctypes.POINTER(ModelDesc), ctypes.POINTER(TensorView), I, ctypes.POINTER(P)], I),
        "ijb_destroy": ([P], None),
        "ijb_last_error": ([P], ctypes.c_char_p),
        "ijb_tensor_index": ([P, ctypes.c_char_p], I),
        "ijb_matvec": ([P, I, P, P, I, I, I, P], I),
        "ijb_forward": ([P, I, I, I, IP], I),
        "ijb_prefill": ([P, IP, I, IP], I),
        "ijb_reset": ([P], I),
        "ijb_logits_dev": ([P], P),
        "ijb_residual_dev": ([P], P),
        "ijb_seq_open": ([P, IP], I),
        "ijb_seq_close": ([P, I], I),
        "ijb_seq_length": ([P, I], I),
        "ijb_decode_step": ([P, I, IP, IP, IP], I),
        "ijb_generate": ([P, I, I, I, IP, I, IP, IP], I),
        "ijb_seq_prefill": ([P, I, IP, I, IP], I),
        "ijb_argmax": ([P, I, P, P], I),
        "ijb_argmax_noalloc": ([P, I, P, P], I),
        "ijb_dequant": ([I, P, L64, P, P], I),
        "ijb_q6k_planar_row_bytes": ([I], L64),
        "ijb_repack_q6k": ([P, P, I, I, P], I),
        "ijb_gemv": ([I, P, P, P, I, I, I, I, P], I),
        "ijb_probe_wait_timeout": ([P, ctypes.c_uint64], I),
        "ijb_forward_traced": ([P, I, I, I, IP, P, P], I),
        "ijb_prefill_traced": ([P, IP, I, IP, P, P, P], I),
        "ijb_last_step_size": ([P], I),
        "ijb_time_layer_projections": ([P, I, I, ctypes.POINTER(ctypes.c_float)], I),
        "ijb_time_layer_attention": ([P, I, IP, I, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_longlong)], I),
        "ijb_weight_create": ([I, P, I, I, I, ctypes.POINTER(P)], I),
        "ijb_weight_destroy": ([P], None),
        "ijb_weight_matmul": ([P, P, I, P, ctypes.c_float, I, P, L64, I, P, P], I),
        "ijb_weight_status": ([P], I),
        "ijb_keys_to_tokens": ([P, I, P, P], I),
        "ijb_kernel_launches": ([], ctypes.c_uint64),
        "ijb_tokenizer_create": ([ctypes.POINTER(ctypes.c_char_p), I, ctypes.POINTER(ctypes.c_char_p), I,
                                  ctypes.POINTER(P)], I),
        "ijb_tokenizer_destroy": ([P], None),
        "ijb_tokenizer_last_error": ([P], ctypes.c_char_p),
        "ijb_tokenizer_encode": ([P, ctypes.c_char_p, L64, IP, L64, ctypes.POINTER(L64)], I),
        "ijb_tokenizer_decode": ([P, I, ctypes.c_char_p, I, IP], I),
        "ijb_tokenizer_special": ([P, ctypes.c_char_p, IP], I),
        "ijb_tokenizer_chat_prompt": ([P, ctypes.c_char_p, L64, IP, L64, ctypes.POINTER(L64)], I),
        "ijb_tokenizer_encode_batch": ([P, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(L64), I, IP, L64,
                                        ctypes.POINTER(L64), I], I),
        "ijb_last_step_ms": ([P], ctypes.c_float),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def declared_symbols() -> list[str]:
    """Every function include/ijb200.h declares."""
    import re
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ijb_[a-z0-9_]+)\s*\(", text)))


def check(rc: int, engine=None) -> None:
    if rc != OK:
        msg = load().ijb_last_error(engine)
        raise IjbError(rc, msg.decode() if msg else "")
