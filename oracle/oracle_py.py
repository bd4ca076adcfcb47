"""ctypes access to the oracle (liboracle.so) and to the reference builds in
oracle/_ref/.  TEST INFRASTRUCTURE ONLY: imported by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline / reference arm, and
only as the checker or the timed CPU baseline.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
VOCAB_SIZE = 151936
FP32, BF16, FP32_KV = 0, 1, 2

_lib = None


def lib():
    global _lib
    if _lib is None:
        p = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(p):
            raise RuntimeError("oracle not built: run oracle/build_oracle.py")
        L = ctypes.CDLL(p)
        vp, c = ctypes.c_void_p, ctypes
        L.oracle_open.argtypes = [c.c_char_p, c.c_int, c.c_int, c.POINTER(vp)]
        L.oracle_close.argtypes = [vp]
        L.oracle_forward.argtypes = [vp, c.c_int, c.c_int, vp, vp]
        L.oracle_set_dump.argtypes = [vp, vp]
        L.oracle_set_dump_qkv.argtypes = [vp, vp]
        L.oracle_set_float_accum.argtypes = [vp, c.c_int]
        L.oracle_fill_kv.argtypes = [vp, c.c_int, c.c_ulonglong]
        L.oracle_set_ref_softmax.argtypes = [vp, c.c_int]
        L.oracle_set_threads.argtypes = [c.c_int]
        L.oracle_get_threads.restype = c.c_int
        L.oracle_gemv_bf16.argtypes = [vp, vp, vp, c.c_int, c.c_int]
        L.oracle_sample.argtypes = [vp, c.c_int, c.c_float, c.c_float, c.c_int, c.POINTER(c.c_ulonglong), c.c_int]
        L.oracle_random_u32.argtypes = [c.POINTER(c.c_ulonglong)]
        L.oracle_random_u32.restype = c.c_uint
        L.oracle_rope_cs.argtypes = [c.c_int, c.c_int, c.POINTER(c.c_float), c.POINTER(c.c_float)]
        L.oracle_write_synthetic.argtypes = [c.c_char_p, c.c_ulonglong]
        _lib = L
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def write_synthetic_checkpoint(path, seed=0):
    """The seed-`seed` synthetic safetensors checkpoint, written by the oracle
    (byte-identical to the library's own writer; bench.py's reference arm uses
    this so that it never loads the product library)."""
    if lib().oracle_write_synthetic(path.encode(), int(seed)) != 0:
        raise RuntimeError(f"oracle_write_synthetic failed for {path}")


def set_threads(n):
    lib().oracle_set_threads(int(n))


def get_threads():
    return lib().oracle_get_threads()


class Oracle:
    """CPU restatement of forward(token, pos) (mode FP32 or BF16)."""

    def __init__(self, checkpoint, mode=FP32, max_seq=1024):
        h = ctypes.c_void_p()
        rc = lib().oracle_open(checkpoint.encode(), mode, max_seq, ctypes.byref(h))
        if rc != 0:
            raise RuntimeError(f"oracle_open failed ({rc})")
        self._h = h
        self.mode = mode

    def fill_kv(self, n, seed=1):
        """Populate cache positions [0, n) with seeded values (timing runs only)."""
        if lib().oracle_fill_kv(self._h, int(n), int(seed)) != 0:
            raise RuntimeError("oracle_fill_kv failed")

    def set_ref_softmax(self, on):
        """bf16 mode: reproduce the reference's softmax reduction, dropped terms included."""
        lib().oracle_set_ref_softmax(self._h, 1 if on else 0)

    def set_float_accum(self, on):
        lib().oracle_set_float_accum(self._h, 1 if on else 0)

    def close(self):
        if self._h:
            lib().oracle_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, token, pos, want_logits=True, want_xfinal=False, dump=None, dump_qkv=None):
        lg = np.zeros(VOCAB_SIZE, dtype=np.float32) if want_logits else None
        xf = np.zeros(1024, dtype=np.float32) if want_xfinal else None
        if dump is not None:
            lib().oracle_set_dump(self._h, _p(dump))
        if dump_qkv is not None:
            lib().oracle_set_dump_qkv(self._h, _p(dump_qkv))
        rc = lib().oracle_forward(self._h, int(token), int(pos), _p(lg) if lg is not None else None,
                                  _p(xf) if xf is not None else None)
        if dump is not None:
            lib().oracle_set_dump(self._h, None)
        if dump_qkv is not None:
            lib().oracle_set_dump_qkv(self._h, None)
        if rc != 0:
            raise RuntimeError(f"oracle_forward failed ({rc})")
        if want_xfinal:
            return lg, xf
        return lg


def gemv_bf16(W, x):
    """W uint16 [n][k] (bf16 bits), x uint16 [k] -> y uint16 [n]."""
    W = np.ascontiguousarray(W, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.zeros(W.shape[0], dtype=np.uint16)
    lib().oracle_gemv_bf16(_p(W), _p(x), _p(y), W.shape[0], W.shape[1])
    return y


def sample(logits, temperature, topp, top_k, rng, order_mode=0):
    """Returns (token, new rng).  order_mode 0: the reference's candidate order;
    1: descending probability, ties by ascending id (the device sampler)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    r = ctypes.c_ulonglong(rng)
    t = lib().oracle_sample(_p(lg), lg.size, temperature, topp, top_k, ctypes.byref(r), order_mode)
    return t, r.value


def rope_cs(pos, j):
    c, s = ctypes.c_float(), ctypes.c_float()
    lib().oracle_rope_cs(pos, j, ctypes.byref(c), ctypes.byref(s))
    return c.value, s.value


# ---- the reference's own code, built into oracle/_ref/ ----------------------
def ref_sampler():
    p = os.path.join(HERE, "_ref", "libref_sampler.so")
    if not os.path.exists(p):
        return None
    L = ctypes.CDLL(p)
    L.ref_sample.argtypes = [ctypes.c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.POINTER(ctypes.c_ulonglong)]
    L.ref_sample.restype = ctypes.c_int
    return L


def ref_model():
    p = os.path.join(HERE, "_ref", "libref_model.so")
    if not os.path.exists(p):
        return None
    L = ctypes.CDLL(p)
    L.ref_build.argtypes = [ctypes.c_char_p]
    L.ref_forward.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return L


def bf16_bits(a):
    """float32 array -> bf16 bit patterns (round to nearest even)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
