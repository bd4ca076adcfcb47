"""Python bindings of libqwen_b200.so (the C ABI declared in include/qwen_b200.h).

The engine is the shared library; this module only declares argument types,
turns status codes into exceptions and moves numpy arrays across.  It never
computes model math itself: if the library is missing, loading fails loudly.

Reference counterparts (Ramshankar07/qwen600-ROCm-inference):
  Engine(...)              build_transformer   qwen_model.cuh:82-92
  Engine.forward           forward             qwen_model.cuh:772-851
  Engine.decode_step       forward + sample    main.cu:144-145, sampler.h:120-175
  Engine.close             free_transformer    qwen_model.cuh:94-111
  sample_host              sample              sampler.h:120-175
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "lib", "libqwen_b200.so")

VOCAB_SIZE = 151936
DIM = 1024
SEQ_LEN = 8192
N_LAYERS = 28

QWEN_OK = 0
STATUS = {-1: "QWEN_E_ARG", -2: "QWEN_E_IO", -3: "QWEN_E_FORMAT", -4: "QWEN_E_CUDA", -5: "QWEN_E_TIMEOUT",
          -6: "QWEN_E_UNSUPPORTED", -7: "QWEN_E_STATE"}

# every entry point of include/qwen_b200.h: name -> (restype, argtypes)
_c = ctypes
_P = _c.c_void_p
_SIGS = {
    "qwen_last_error": (_c.c_char_p, []),
    "qwen_abi_version": (_c.c_int, []),
    "qwen_num_tensors": (_c.c_int, []),
    "qwen_vocab_size": (_c.c_int, []),
    "qwen_total_weight_bytes": (_c.c_size_t, []),
    "qwen_tensor_info": (_c.c_int, [_c.c_int, _c.POINTER(_c.c_char_p), _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t)]),
    "qwen_checkpoint_validate": (_c.c_int, [_c.c_char_p]),
    "qwen_weights_load": (_c.c_int, [_c.c_char_p, _c.c_int, _c.POINTER(_P)]),
    "qwen_weights_free": (_c.c_int, [_P]),
    "qwen_write_synthetic_checkpoint": (_c.c_int, [_c.c_char_p, _c.c_uint64]),
    "qwen_write_ordered_blob": (_c.c_int, [_c.c_char_p, _c.c_char_p]),
    "qwen_create": (_c.c_int, [_c.c_char_p, _c.c_int, _c.POINTER(_P)]),
    "qwen_destroy": (None, [_P]),
    "qwen_device": (_c.c_int, [_P]),
    "qwen_forward": (_c.c_int, [_P, _c.c_int, _c.c_int, _P]),
    "qwen_host_logits": (_P, [_P]),
    "qwen_device_logits": (_P, [_P]),
    "qwen_device_weights": (_P, [_P]),
    "qwen_read_logits": (_c.c_int, [_P, _P]),
    "qwen_decode_step": (_c.c_int, [_P, _c.c_int, _c.c_int, _P, _c.POINTER(_c.c_ulonglong), _c.POINTER(_c.c_int)]),
    "qwen_generate": (_c.c_int, [_P, _c.c_int, _c.c_int, _c.c_int, _P, _c.POINTER(_c.c_ulonglong), _P]),
    "qwen_generate_timed": (_c.c_int, [_P, _c.c_int, _c.c_int, _c.c_int, _P, _c.POINTER(_c.c_ulonglong), _P,
                                       _c.POINTER(_c.c_float)]),
    "qwen_prefill": (_c.c_int, [_P, _P, _c.c_int, _c.c_int, _P]),
    "qwen_cached_positions": (_c.c_int, [_P]),
    "qwen_set_vocab_shard": (_c.c_int, [_P, _c.c_int, _c.c_int]),
    "qwen_shard_topk": (_c.c_int, [_P, _c.c_int, _P, _P]),
    "qwen_stream": (_P, [_P]),
    "qwen_shard_begin": (_c.c_int, [_P, _c.c_int, _c.c_int, _P, _c.c_ulonglong]),
    "qwen_shard_decode": (_c.c_int, [_P]),
    "qwen_shard_candidates": (_c.c_int, [_P, _P, _P]),
    "qwen_shard_merge": (_c.c_int, [_P, _P, _P, _c.c_int, _c.c_int]),
    "qwen_shard_finish": (_c.c_int, [_P, _P, _c.c_int, _c.POINTER(_c.c_ulonglong)]),
    "qwen_sample_host": (_c.c_int, [_P, _c.c_int, _P, _c.POINTER(_c.c_ulonglong), _c.POINTER(_c.c_int)]),
    "qwen_sample_candidates": (_c.c_int, [_P, _P, _c.c_int, _P, _c.POINTER(_c.c_ulonglong), _c.POINTER(_c.c_int)]),
    "qwen_debug_chunk_counts": (_c.c_int, [_P, _P, _c.c_int]),
    "qwen_debug_capture": (_c.c_int, [_P, _c.c_int]),
    "qwen_debug_read": (_c.c_int, [_P, _P, _P]),
    "qwen_trace_enable": (_c.c_int, [_P, _c.c_int]),
    "qwen_debug_inject_wait": (_c.c_int, [_P, _c.c_ulonglong, _c.c_int]),
    "qwen_trace_read": (_c.c_int, [_P, _P, _c.c_int]),
    "qwen_gemv_bf16": (_c.c_int, [_P, _P, _P, _c.c_int, _c.c_int, _P]),
    "qwen_gemv_bf16_static": (_c.c_int, [_P, _P, _P, _c.c_int, _c.c_int, _P]),
    "qwen_gemv_bf16_status": (_c.c_int, [_P]),
    "qwen_gemv_bf16_static_status": (_c.c_int, [_P]),
    "qwen_gemm_bf16": (_c.c_int, [_P, _P, _P, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _P]),
    "qwen_set_prefill_mode": (_c.c_int, [_P, _c.c_int]),
    "qwen_set_prefill_parts": (_c.c_int, [_P, _c.c_int]),
    "qwen_set_prefill_attention": (_c.c_int, [_P, _c.c_int]),
    "qwen_row_topk": (_c.c_int, [_P, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _P, _P, _P]),
    "qwen_batch_init": (_c.c_int, [_P, _c.c_int]),
    "qwen_batch_prefill": (_c.c_int, [_P, _c.c_int, _P, _c.c_int, _P]),
    "qwen_batch_step": (_c.c_int, [_P, _c.c_int, _P, _P, _P, _P, _P]),
    "qwen_batch_read_logits": (_c.c_int, [_P, _c.c_int, _P]),
    "qwen_tokenizer_load": (_c.c_int, [_c.c_char_p, _c.c_int, _c.POINTER(_P)]),
    "qwen_tokenizer_free": (None, [_P]),
    "qwen_tokenizer_info": (_c.c_int, [_P, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int), _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)]),
    "qwen_tokenizer_encode": (_c.c_int, [_P, _c.c_char_p, _P, _c.c_int, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)]),
    "qwen_tokenizer_decode": (_c.c_int, [_P, _c.c_int, _c.POINTER(_c.c_char_p)]),
}

_lib = None


class QwenError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class Sampling(ctypes.Structure):
    """qwen_sampling_t: temperature, top-p, top-k (sampler.h:17-24)."""
    _fields_ = [("temperature", ctypes.c_float), ("topp", ctypes.c_float), ("top_k", ctypes.c_int)]


GREEDY = Sampling(0.0, 1.0, 1)


def load_library(path=None):
    """Load the engine library; raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"engine library not built: {p} (run qwen600-rocm-inference_b200/build.py)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in _SIGS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _lib = lib
    return lib


def _check(rc):
    if rc != QWEN_OK:
        raise QwenError(rc, load_library().qwen_last_error().decode())


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def tensor_table():
    """[(name, offset, bytes)] of the canonical weight layout."""
    lib = load_library()
    out = []
    for i in range(lib.qwen_num_tensors()):
        n, o, b = ctypes.c_char_p(), ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib.qwen_tensor_info(i, ctypes.byref(n), ctypes.byref(o), ctypes.byref(b)))
        out.append((n.value.decode(), o.value, b.value))
    return out


def checkpoint_validate(path):
    _check(load_library().qwen_checkpoint_validate(path.encode()))


def write_ordered_blob(safetensors_path, out_path):
    """The reference's weights_qwen600.bin (export.py:80-146) of a BF16 safetensors checkpoint."""
    _check(load_library().qwen_write_ordered_blob(safetensors_path.encode(), out_path.encode()))


def write_synthetic_checkpoint(path, seed=0):
    _check(load_library().qwen_write_synthetic_checkpoint(path.encode(), seed))


def default_checkpoint(seed=0, directory=None):
    """Path of the seed-`seed` synthetic checkpoint, written on first use.

    Several processes may ask at once (one per GPU under torchrun): each writes
    its own temporary file and renames it into place, so no process ever maps
    a file that another is still writing (the rename is atomic; a mapping of
    the replaced file stays valid)."""
    d = directory or os.environ.get("QWEN_B200_CACHE", os.path.join(REPO, ".cache"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"qwen3-0.6b-synthetic-seed{seed}.safetensors")
    if not os.path.exists(path):
        tmp = f"{path}.tmp.{os.getpid()}"
        try:
            write_synthetic_checkpoint(tmp, seed)
            os.replace(tmp, path)
        finally:
            if os.path.exists(tmp):
                os.remove(tmp)
    return path


def sample_host(logits, sampling, rng):
    """sampler.h sample() on host logits; returns (token, new rng state)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    r = ctypes.c_ulonglong(rng)
    t = ctypes.c_int()
    _check(load_library().qwen_sample_host(_ptr(lg), lg.size, ctypes.byref(sampling), ctypes.byref(r), ctypes.byref(t)))
    return t.value, r.value


def sample_candidates(values, ids, sampling, rng):
    v = np.ascontiguousarray(values, dtype=np.float32)
    i = np.ascontiguousarray(ids, dtype=np.int32)
    r = ctypes.c_ulonglong(rng)
    t = ctypes.c_int()
    _check(load_library().qwen_sample_candidates(_ptr(v), _ptr(i), v.size, ctypes.byref(sampling), ctypes.byref(r),
                                                 ctypes.byref(t)))
    return t.value, r.value


def gemv_bf16(W_ptr, x_ptr, y_ptr, n, k, stream=0):
    """y = bf16(W x) on device pointers (ints)."""
    _check(load_library().qwen_gemv_bf16(ctypes.c_void_p(W_ptr), ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), n, k,
                                         ctypes.c_void_p(stream)))


def gemv_status(stream=0, static=False):
    """Synchronise `stream`; raise QwenError (QWEN_E_TIMEOUT) if a GEMV launch of
    the chosen entry point since the last query had a device wait expire."""
    lib = load_library()
    f = lib.qwen_gemv_bf16_static_status if static else lib.qwen_gemv_bf16_status
    _check(f(ctypes.c_void_p(stream)))


def row_topk(logits_ptr, rows, n, ld, k, values_ptr, ids_ptr, stream=0):
    """The k best entries of each row of fp32 logits (device pointers, ints):
    values and column ids, k per row, in column order."""
    _check(load_library().qwen_row_topk(ctypes.c_void_p(logits_ptr), rows, n, ld, k, ctypes.c_void_p(values_ptr),
                                         ctypes.c_void_p(ids_ptr), ctypes.c_void_p(stream)))


def gemm_bf16(A_ptr, B_ptr, C_ptr, M, N, K, c_fp32=True, stream=0):
    """C = A B^T on device pointers (ints): A [M][K] bf16, B [N][K] bf16, C [M][N] fp32 or bf16."""
    _check(load_library().qwen_gemm_bf16(ctypes.c_void_p(A_ptr), ctypes.c_void_p(B_ptr), ctypes.c_void_p(C_ptr), M, N, K,
                                         1 if c_fp32 else 0, ctypes.c_void_p(stream)))


def gemv_bf16_static(W_ptr, x_ptr, y_ptr, n, k, stream=0):
    """y = bf16(W x) on device pointers, without any device allocation."""
    _check(load_library().qwen_gemv_bf16_static(ctypes.c_void_p(W_ptr), ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), n, k,
                                                ctypes.c_void_p(stream)))


class Engine:
    """One model instance on one GPU (a qwen_t handle)."""

    def __init__(self, checkpoint, device=0):
        self._lib = load_library()
        h = ctypes.c_void_p()
        _check(self._lib.qwen_create(checkpoint.encode(), device, ctypes.byref(h)))
        self._h = h
        self.device = device
        self._host_logits = self._lib.qwen_host_logits(h)

    def close(self):
        if self._h:
            self._lib.qwen_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def cached(self):
        return self._lib.qwen_cached_positions(self._h)

    def forward(self, token, pos, want_logits=True):
        """forward(token, pos): returns a copy of the VOCAB_SIZE fp32 logits (or None)."""
        _check(self._lib.qwen_forward(self._h, int(token), int(pos), ctypes.c_void_p(self._host_logits) if want_logits else None))
        if not want_logits:
            return None
        buf = (ctypes.c_float * VOCAB_SIZE).from_address(self._host_logits)
        return np.frombuffer(buf, dtype=np.float32).copy()

    def forward_into(self, token, pos, out):
        """forward with the logits copied straight into `out` (float32 host array)."""
        _check(self._lib.qwen_forward(self._h, int(token), int(pos), _ptr(out)))

    def read_logits(self):
        """fp32 logits of the last step (all rows this handle serves)."""
        out = np.zeros(VOCAB_SIZE, dtype=np.float32)
        n = self._lib.qwen_read_logits(self._h, _ptr(out))
        if n < 0:
            _check(n)
        return out[:n]

    def device_logits_ptr(self):
        return self._lib.qwen_device_logits(self._h)

    def decode_step(self, token, pos, sampling=GREEDY, rng=0):
        r = ctypes.c_ulonglong(rng)
        t = ctypes.c_int()
        _check(self._lib.qwen_decode_step(self._h, int(token), int(pos), ctypes.byref(sampling), ctypes.byref(r), ctypes.byref(t)))
        return t.value, r.value

    def generate(self, token, pos, n_steps, sampling=GREEDY, rng=0):
        out = np.zeros(n_steps, dtype=np.int32)
        r = ctypes.c_ulonglong(rng)
        _check(self._lib.qwen_generate(self._h, int(token), int(pos), int(n_steps), ctypes.byref(sampling), ctypes.byref(r), _ptr(out)))
        return out.tolist(), r.value

    def generate_timed(self, token, pos, n_steps, sampling=GREEDY, rng=0):
        """generate() plus the device time (ms) of its launches, from CUDA events."""
        out = np.zeros(n_steps, dtype=np.int32)
        r = ctypes.c_ulonglong(rng)
        ms = ctypes.c_float()
        _check(self._lib.qwen_generate_timed(self._h, int(token), int(pos), int(n_steps), ctypes.byref(sampling), ctypes.byref(r),
                                             _ptr(out), ctypes.byref(ms)))
        return out.tolist(), r.value, ms.value

    # ---- batched decode (qwen_batch_*) ----
    def batch_init(self, max_batch):
        _check(self._lib.qwen_batch_init(self._h, int(max_batch)))

    def batch_prefill(self, slot, tokens, want_logits=False):
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(VOCAB_SIZE, dtype=np.float32) if want_logits else None
        _check(self._lib.qwen_batch_prefill(self._h, int(slot), _ptr(tk), tk.size, _ptr(lg) if want_logits else None))
        return lg

    def batch_step(self, tokens, positions, sampling=GREEDY, rng_states=None):
        """One step for slots 0 .. len(tokens)-1; returns (next tokens, rng states)."""
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        ps = np.ascontiguousarray(positions, dtype=np.int32)
        nx = np.zeros(tk.size, dtype=np.int32)
        rs = None if rng_states is None else np.ascontiguousarray(rng_states, dtype=np.uint64)
        _check(self._lib.qwen_batch_step(self._h, tk.size, _ptr(tk), _ptr(ps), ctypes.byref(sampling),
                                         _ptr(rs) if rs is not None else None, _ptr(nx)))
        return nx.tolist(), (rs.tolist() if rs is not None else None)

    def batch_read_logits(self, rows):
        """fp32 logits of the last batch_step's first `rows` rows, shape (rows, VOCAB_SIZE)."""
        out = np.zeros((int(rows), VOCAB_SIZE), dtype=np.float32)
        _check(self._lib.qwen_batch_read_logits(self._h, int(rows), _ptr(out)))
        return out

    def set_prefill_parts(self, parts=3):
        """bf16 parts per activation in the tensor-core passes (3: fp32-exact, 2, 1)."""
        _check(self._lib.qwen_set_prefill_parts(self._h, int(parts)))

    def set_prefill_attention(self, kind=1):
        """Prompt-pass attention kernel: 1 tcgen05/TMEM (default, one pass over the
        keys with an online softmax), 0 mma.sync."""
        _check(self._lib.qwen_set_prefill_attention(self._h, int(kind)))

    def set_prefill_mode(self, gemm=True):
        """Long prompts on the tensor cores (True, default) or one decode launch per token."""
        _check(self._lib.qwen_set_prefill_mode(self._h, 1 if gemm else 0))

    def prefill(self, tokens, pos0=0, want_logits=False):
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        lg = np.zeros(VOCAB_SIZE, dtype=np.float32) if want_logits else None
        _check(self._lib.qwen_prefill(self._h, _ptr(tk), tk.size, int(pos0), _ptr(lg) if want_logits else None))
        return lg

    def chunk_counts(self):
        out = np.zeros(2 * 1024, dtype=np.int32)
        n = self._lib.qwen_debug_chunk_counts(self._h, _ptr(out), 1024)
        if n < 0:
            _check(n)
        return out[: 2 * n].reshape(n, 2)

    def debug_capture(self, enable=True):
        _check(self._lib.qwen_debug_capture(self._h, 1 if enable else 0))

    def debug_read(self):
        """(residual after each layer [28,1024], raw q|k|v projections [28,4096]) of the last launch."""
        r = np.zeros((N_LAYERS, DIM), dtype=np.float32)
        q = np.zeros((N_LAYERS, 4096), dtype=np.float32)
        _check(self._lib.qwen_debug_read(self._h, _ptr(r), _ptr(q)))
        return r, q

    TRACE_STRIDE = 576

    def debug_inject_wait(self, wait_ns=0, group=-1):
        """Failure testing: wait limit for later launches (0 = default) and a KV
        head whose CTAs withhold their layer-0 q|k|v (-1 = none)."""
        _check(self._lib.qwen_debug_inject_wait(self._h, int(wait_ns), int(group)))

    def trace_enable(self, enable=True):
        _check(self._lib.qwen_trace_enable(self._h, 1 if enable else 0))

    def trace_read(self):
        """[n_ctas, TRACE_STRIDE] %globaltimer stamps (ns) of the last launch."""
        out = np.zeros(1024 * self.TRACE_STRIDE, dtype=np.uint64)
        n = self._lib.qwen_trace_read(self._h, _ptr(out), out.size)
        if n < 0:
            _check(n)
        return out[:n].reshape(-1, self.TRACE_STRIDE)

    # ---- device-resident sharded head (see sharding.py) ----
    @property
    def stream(self):
        """The handle's cudaStream_t (an int), for work that must follow its launches."""
        return self._lib.qwen_stream(self._h) or 0

    def shard_begin(self, token, pos, sampling=GREEDY, rng=0):
        k = self._lib.qwen_shard_begin(self._h, int(token), int(pos), ctypes.byref(sampling), int(rng))
        if k < 0:
            _check(k)
        return k

    def shard_decode(self):
        _check(self._lib.qwen_shard_decode(self._h))

    def shard_candidates(self, values_ptr, ids_ptr):
        _check(self._lib.qwen_shard_candidates(self._h, ctypes.c_void_p(values_ptr), ctypes.c_void_p(ids_ptr)))

    def shard_merge(self, values_ptr, ids_ptr, n_ranks, stride):
        _check(self._lib.qwen_shard_merge(self._h, ctypes.c_void_p(values_ptr), ctypes.c_void_p(ids_ptr), int(n_ranks), int(stride)))

    def shard_finish(self, n):
        toks = np.zeros(max(int(n), 1), dtype=np.int32)
        r = ctypes.c_ulonglong()
        _check(self._lib.qwen_shard_finish(self._h, _ptr(toks), int(n), ctypes.byref(r)))
        return toks[:n].tolist(), r.value

    def set_vocab_shard(self, begin, end):
        _check(self._lib.qwen_set_vocab_shard(self._h, int(begin), int(end)))

    def shard_topk(self, k):
        v = np.zeros(k, dtype=np.float32)
        i = np.zeros(k, dtype=np.int32)
        _check(self._lib.qwen_shard_topk(self._h, int(k), _ptr(v), _ptr(i)))
        return v, i
