"""Python binding of libvarda_b200 (include/varda_b200.h) through ctypes.

Mirrors the reference's public C++ API (varda.cpp src/varda/varda.h:21-76): Options, Model.load,
Model.predict_step(x, y, hook), plus the CudaBackend device entry points and the kernel-level entry
points used by the tests. The shared library must exist (built by `make -C varda.cpp_b200`); there is
no fallback: every call goes to the CUDA library, and a missing library raises ImportError. The library
is loaded on the first call that needs it, so the pure-Python modules of the package (`synth`,
`safetensors`) import without it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvarda_b200.so")

FP32, FP16 = 0, 1
ERRORS = {1: "invalid argument", 2: "format", 3: "cuda", 4: "unsupported", 5: "internal", 6: "timeout"}


class VardaError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{ERRORS.get(code, code)}] {msg}")
        self.code = code


def _load_lib():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C varda.cpp_b200`")
    L = ctypes.CDLL(LIB_PATH)
    P, I, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    sig = {
        "vb_last_error": ([], ctypes.c_char_p),
        "vb_load": ([ctypes.c_char_p, P, P], I),
        "vb_load_sharded": ([ctypes.c_char_p, P, I, I, P, P], I),
        "vb_nccl_unique_id": ([P], I),
        "vb_free": ([P], None),
        "vb_predict_step": ([P, P, P, P, P], I),
        "vb_sizes": ([P, P], I),
        "vb_data_range": ([P, P, P], I),
        "vb_io_numel": ([P, P, P], I),
        "vb_normalise": ([P, P, P, P], I),
        "vb_forward_normalised": ([P, P, P, P], I),
        "vb_denormalise": ([P, P, P, P], I),
        "vb_predict_step_device": ([P, P, P, P], I),
        "vb_prepare": ([P], I),
        "vb_use_high_priority_stream": ([P], I),
        "vb_device_input": ([P], P),
        "vb_device_output": ([P], P),
        "vb_stream": ([P], P),
        "vb_enqueue_predict": ([P], I),
        "vb_device": ([P], I),
        "vb_weight_bytes": ([P], SZ),
        "vb_activation_bytes": ([P], SZ),
        "vb_decoder_chunk_rows": ([P], I64),
        "vb_check_device": ([], I),
        "vb_launch_count": ([], I64),
        "vb_shard_plan": ([ctypes.c_char_p, I, I, ctypes.c_char_p, SZ], I64),
        "vb_profile_forward": ([P, ctypes.c_char_p, SZ], I64),
        "vb_hidden_range": ([P, P, P], I),
        "vb_processor_block": ([P, I, P, P, I, P], I),
        "vb_profile_processor_block": ([P, I, ctypes.c_char_p, SZ], I64),
        "vb_build_csr": ([P, I64, P, I, I64, I64, P, P, P, P], I),
        "vb_pack_edges": ([P, P, I, I64, I, P], I),
        "vb_attention": ([I, P, P, I64, I64, P, I64, P, P, I64, P, I64, P, I64, P, I, I, I, P], I),
        "vb_gemm": ([I, I, P, I64, P, I64, P, P, I64, P, I64, I64, I64, I64, I, I, P], I),
        "vb_layernorm": ([I, P, I64, P, P, P, I64, I64, I, F, P], I),
        "vb_ln_segment_width": ([I64], I),
        "vb_gemm_ln": ([P, I64, P, I64, P, P, I64, P, I64, I64, I64, I64, I, I, P, P, P, I, I, F, P], I),
        "vb_fold_layernorm": ([P, I64, I64, I, P, P, P, P, P], I),
        "vb_row_seg_stats": ([P, I64, I64, I, I, P, P], I),
        "vb_add_layernorm": ([I, P, P, P, P, P, P, I64, I64, I, F, P], I),
        "vb_rollout": ([P, P, I, P, P, I, P, P, P], I),
        "vb_attention_rows": ([I, P, P, P, I64, P, I64, P, P, I64, P, I64, P, I64, P, I, I, I, P], I),
        "vb_attention_split_noalloc": ([I, P, P, I64, I64, P, I64, P, P, I64, P, I64, P, I64, P, I, I, I, I, P], I),
        "vb_rollout_update": ([P, I, I64, I, P, P, I64, I, P, I, P, P, P], I),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _bind_tiles(L)
    return L


class _LazyLib:
    """The ctypes handle of libvarda_b200, opened (and its signatures bound) on first attribute access."""

    _handle = None

    def get(self):
        if _LazyLib._handle is None:
            _LazyLib._handle = _load_lib()
        return _LazyLib._handle

    def __getattr__(self, name):
        return getattr(self.get(), name)


lib = _LazyLib()


def __getattr__(name):
    # exported symbols, for the ABI check in the tests (opens the library)
    if name == "SYMBOLS":
        return [n for n in dir(lib.get()) if n.startswith("vb_")]
    raise AttributeError(name)


def check(rc):
    if rc != 0:
        raise VardaError(rc, lib.vb_last_error().decode(errors="replace"))


class Options(ctypes.Structure):
    """varda::Options (varda.h:21-27)."""
    _fields_ = [("precision", ctypes.c_int), ("cuda_device", ctypes.c_int), ("cuda_graph", ctypes.c_int),
                ("num_threads", ctypes.c_int)]


HOOK = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int64),
                        ctypes.c_int, ctypes.c_void_p)
STEP = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_int64, ctypes.c_void_p)


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return ctypes.c_void_p(a)
    if hasattr(a, "data_ptr"):  # torch tensor (device memory plumbing)
        return ctypes.c_void_p(a.data_ptr())
    return a.ctypes.data_as(ctypes.c_void_p)


def _check_out(a, n, what):
    """An output array the library writes through a raw pointer: fp32, C-contiguous, writable, n elements."""
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous or not a.flags.writeable:
        raise ValueError(f"{what} must be a writable C-contiguous float32 numpy array")
    if a.size != n:
        raise ValueError(f"{what} has {a.size} elements, expected {n}")


class Model:
    """varda::Model (varda.h:37-76) on the B200 backend."""

    def __init__(self, handle, path=None):
        self._h = handle
        self._path = path
        s = (ctypes.c_int64 * 8)()
        check(lib.vb_sizes(self._h, s))
        self.T_in, self.G, self.V_in, self.T_out, self.V_out, self.H, self.C, self.n_proc = list(s)
        lo, hi = ctypes.c_int64(), ctypes.c_int64()
        check(lib.vb_data_range(self._h, ctypes.byref(lo), ctypes.byref(hi)))
        self.data_lo, self.data_hi = lo.value, hi.value
        check(lib.vb_hidden_range(self._h, ctypes.byref(lo), ctypes.byref(hi)))
        self.hidden_lo, self.hidden_hi = lo.value, hi.value
        i, o = ctypes.c_int64(), ctypes.c_int64()
        check(lib.vb_io_numel(self._h, ctypes.byref(i), ctypes.byref(o)))
        self.device_input_numel, self.device_output_numel = i.value, o.value

    @staticmethod
    def load(path, precision=FP16, cuda_device=0, cuda_graph=True):
        o = Options(precision, cuda_device, int(cuda_graph), 0)
        h = ctypes.c_void_p()
        check(lib.vb_load(os.fsencode(path), ctypes.byref(o), ctypes.byref(h)))
        return Model(h, path)

    @staticmethod
    def load_sharded(path, rank, world, nccl_id, precision=FP16, cuda_device=0, cuda_graph=True):
        o = Options(precision, cuda_device, int(cuda_graph), 0)
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        check(lib.vb_load_sharded(os.fsencode(path), ctypes.byref(o), rank, world, buf, ctypes.byref(h)))
        return Model(h, path)

    def free(self):
        if self._h:
            lib.vb_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def input_shape(self):
        return (1, self.T_in, self.G, self.V_in)

    @property
    def output_shape(self):
        return (1, self.T_out, 1, self.G, self.V_out)

    def predict_step(self, x, y=None, hook=None):
        """Host x (1, T_in, G, V_in) fp32 -> y (1, T_out, 1, G, V_out) fp32. hook(key, array)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != int(np.prod(self.input_shape)):
            raise ValueError(f"x has {x.size} elements, expected {self.input_shape}")
        if y is None:
            y = np.empty(self.output_shape, np.float32)
        else:
            _check_out(y, int(np.prod(self.output_shape)), "y")
        cb = None
        if hook is not None:
            def _cb(key, data, shape, ndim, user):
                shp = tuple(shape[i] for i in range(ndim))
                n = int(np.prod(shp)) if shp else 1
                arr = np.ctypeslib.as_array(data, shape=(n,)).reshape(shp).copy()
                hook(key.decode(), arr)
            cb = HOOK(_cb)
        check(lib.vb_predict_step(self._h, _ptr(x), _ptr(y), cb, None))
        return y

    def rollout(self, x0, n_steps, forcings=None, constants_oldest=False, keep=True, on_step=None):
        """Device rollout with replayed forcings (vb_rollout; DeviceRollout::run, rollout_cuda.cu:160-234).
        x0 (1, T_in, G, V_in); forcings (n_steps - 1, G, F) or None. Returns (y, step_ms) with y
        (n_steps, G, V_out) (this rank's rows filled on a sharded model) or None when keep is False;
        on_step(step, rows_array) gets each step's own rows (a view valid during the call)."""
        x0 = np.ascontiguousarray(x0, dtype=np.float32)
        if x0.size != int(np.prod(self.input_shape)):
            raise ValueError(f"x0 has {x0.size} elements, expected {self.input_shape}")
        f = None if forcings is None else np.ascontiguousarray(forcings, dtype=np.float32)
        G, Vo = self.G, self.V_out
        F = self.n_dynamic_forcings
        if n_steps > 1 and F and f is not None and f.size != (n_steps - 1) * G * F:
            raise ValueError(f"forcings must be ({n_steps - 1}, {G}, {F}) for {n_steps} steps, got {f.shape}")
        y = np.zeros((n_steps, G, Vo), np.float32) if keep else None
        ms = np.zeros(n_steps, np.float32)
        cb = None
        if on_step is not None:
            def _cb(step, data, rows, user):
                on_step(step, np.ctypeslib.as_array(data, shape=(rows * Vo,)).reshape(rows, Vo))
            cb = STEP(_cb)
        check(lib.vb_rollout(self._h, _ptr(x0), n_steps, _ptr(f), _ptr(y), int(constants_oldest), cb, None, _ptr(ms)))
        return y, ms

    @property
    def n_dynamic_forcings(self):
        """F, the number of dynamic forcings a rollout replays (the config's `forcings.dynamic`; 0
        without a forcings section, or when the model's file is not known)."""
        if self._path is None:
            return 0
        import json
        from . import safetensors as st
        cfg = json.loads(st.read(self._path)[1].get("config", "{}"))
        return len(cfg.get("forcings", {}).get("dynamic_input_index", []))

    # CudaBackend device entry points (cuda_backend.h:38-74); pointers are ints / torch tensors
    def normalise(self, x, xn, stream=None):
        check(lib.vb_normalise(self._h, _ptr(x), _ptr(xn), stream))

    def forward_normalised(self, xn, yn, stream=None):
        check(lib.vb_forward_normalised(self._h, _ptr(xn), _ptr(yn), stream))

    def denormalise(self, yn, y, stream=None):
        check(lib.vb_denormalise(self._h, _ptr(yn), _ptr(y), stream))

    def predict_step_device(self, x, y, stream=None):
        check(lib.vb_predict_step_device(self._h, _ptr(x), _ptr(y), stream))

    def prepare(self):
        check(lib.vb_prepare(self._h))

    def enqueue_predict(self):
        check(lib.vb_enqueue_predict(self._h))

    def device_input(self):
        return lib.vb_device_input(self._h)

    def device_output(self):
        return lib.vb_device_output(self._h)

    def stream(self):
        return lib.vb_stream(self._h)

    def profile(self):
        """One eager forward with a CUDA event pair around every launch: list of
        {"name", "ms", "flop", "bytes"} records."""
        return _records(lambda buf, n: lib.vb_profile_forward(self._h, buf, n))

    def processor_block(self, block, z_in=None, z_out=None, repeats=1):
        """The isolated processor block (vb_processor_block): LN_dst then block `block`, `repeats` times on
        the same input, this rank's hidden rows [hidden_lo, hidden_hi). z_in (rows, C) fp32 or None
        (keep the previous call's input); z_out: an array to fill, True for a new one, or None. Returns
        (z_out, device_ms)."""
        rows = self.hidden_hi - self.hidden_lo
        zi = None
        if z_in is not None:
            zi = np.ascontiguousarray(z_in, dtype=np.float32)
            if zi.size != rows * self.C:
                raise ValueError(f"z_in has {zi.size} elements, expected ({rows}, {self.C})")
        if z_out is True:
            z_out = np.empty((rows, self.C), np.float32)
        elif z_out is not None:
            _check_out(z_out, rows * self.C, "z_out")
        ms = ctypes.c_float()
        check(lib.vb_processor_block(self._h, block, _ptr(zi), _ptr(z_out), repeats, ctypes.byref(ms)))
        return z_out, ms.value

    def profile_block(self, block):
        """One run of processor_block(block) on the current block input with a CUDA event pair around
        every launch: records as profile()."""
        return _records(lambda buf, n: lib.vb_profile_processor_block(self._h, block, buf, n))

    @property
    def weight_bytes(self):
        return lib.vb_weight_bytes(self._h)

    @property
    def activation_bytes(self):
        return lib.vb_activation_bytes(self._h)


def _records(call):
    import json
    n = call(None, 0)
    if n < 0:
        check(-n)
    buf = ctypes.create_string_buffer(int(n) + 1024)
    n = call(buf, len(buf))
    if n < 0:
        check(-n)
    return json.loads(buf.value.decode())


# ---------------------------------------------------------------- kernel-level wrappers
def build_csr(edge_index, edge_attr, n_src, n_dst):
    ei = np.ascontiguousarray(edge_index, np.int64)
    ea = np.ascontiguousarray(edge_attr, np.float32)
    E, A = ei.shape[1], ea.shape[1]
    rp = np.empty(n_dst + 1, np.int32)
    src = np.empty(E, np.int32)
    eid = np.empty(E, np.int32)
    at = np.empty((E, A), np.float32)
    check(lib.vb_build_csr(_ptr(ei), E, _ptr(ea), A, n_src, n_dst, _ptr(rp), _ptr(src), _ptr(eid), _ptr(at)))
    return rp, src, eid, at


def pack_edges(src, attr_csr, round_fp16):
    src = np.ascontiguousarray(src, np.int32)
    at = np.ascontiguousarray(attr_csr, np.float32)
    out = np.empty((len(src), 4), np.float32)
    check(lib.vb_pack_edges(_ptr(src), _ptr(at), at.shape[1], len(src), int(round_fp16), _ptr(out)))
    return out


def attention(dtype, row_ptr, edges, dst_lo, n_rows, q, ldq, k, v, ldkv, xr, ldxr, out, ldo, w_e, C, heads,
              head_dim, stream=None):
    check(lib.vb_attention(dtype, _ptr(row_ptr), _ptr(edges), dst_lo, n_rows, _ptr(q), ldq, _ptr(k), _ptr(v), ldkv,
                           _ptr(xr), ldxr, _ptr(out), ldo, _ptr(w_e), C, heads, head_dim, stream))


def attention_rows(dtype, row_ptr, edges, rows, n_rows, q, ldq, k, v, ldkv, xr, ldxr, out, ldo, w_e, C, heads,
                   head_dim, stream=None):
    check(lib.vb_attention_rows(dtype, _ptr(row_ptr), _ptr(edges), _ptr(rows), n_rows, _ptr(q), ldq, _ptr(k), _ptr(v),
                                ldkv, _ptr(xr), ldxr, _ptr(out), ldo, _ptr(w_e), C, heads, head_dim, stream))


def attention_split_noalloc(dtype, row_ptr, edges, dst_lo, n_rows, q, ldq, k, v, ldkv, xr, ldxr, out, ldo, w_e, C,
                            heads, head_dim, splits, stream=None):
    """vb_attention's result through the no-allocation split-row variant (static device scratch)."""
    check(lib.vb_attention_split_noalloc(dtype, _ptr(row_ptr), _ptr(edges), dst_lo, n_rows, _ptr(q), ldq, _ptr(k),
                                         _ptr(v), ldkv, _ptr(xr), ldxr, _ptr(out), ldo, _ptr(w_e), C, heads, head_dim,
                                         splits, stream))


def gemm(dtype, engine, A, lda, W, ldw, bias, Y, ldy, R, ldr, M, N, K, epilogue=0, gelu_tanh=False, stream=None):
    check(lib.vb_gemm(dtype, engine, _ptr(A), lda, _ptr(W), ldw, _ptr(bias), _ptr(Y), ldy, _ptr(R), ldr, M, N, K,
                      epilogue, int(gelu_tanh), stream))


def gemm_ln(A, lda, W, ldw, bias, Y, ldy, R, ldr, M, N, K, epilogue=0, gelu_tanh=False, st_out=None, st_in=None,
            colsum=None, nseg_in=0, segw_in=0, eps=0.0, stream=None):
    """vb_gemm_ln: the fp16 tensor-core GEMM with LayerNorm records written (st_out) or an LN folded in
    (st_in, colsum)."""
    check(lib.vb_gemm_ln(_ptr(A), lda, _ptr(W), ldw, _ptr(bias), _ptr(Y), ldy, _ptr(R), ldr, M, N, K, epilogue,
                         int(gelu_tanh), _ptr(st_out), _ptr(st_in), _ptr(colsum), nseg_in, segw_in, eps, stream))


def fold_layernorm(W, ldw, N, K, g, be, bias, colsum, stream=None):
    check(lib.vb_fold_layernorm(_ptr(W), ldw, N, K, _ptr(g), _ptr(be), _ptr(bias), _ptr(colsum), stream))


def row_seg_stats(x, ldx, rows, C, segw, st, stream=None):
    check(lib.vb_row_seg_stats(_ptr(x), ldx, rows, C, segw, _ptr(st), stream))


def ln_segment_width(N):
    return lib.vb_ln_segment_width(N)


def layernorm(dtype, x, ldx, w, b, y, ldy, rows, C, eps, stream=None):
    check(lib.vb_layernorm(dtype, _ptr(x), ldx, _ptr(w), _ptr(b), _ptr(y), ldy, rows, C, eps, stream))


def add_layernorm(dtype, a, r, out1, w, b, ln, ld, rows, C, eps, stream=None):
    check(lib.vb_add_layernorm(dtype, _ptr(a), _ptr(r), _ptr(out1), _ptr(w), _ptr(b), _ptr(ln), ld, rows, C, eps,
                               stream))


def rollout_update(window, T, rows, V_in, y_own, y_halo, n_own, V_out, f, F, kind, src, stream=None):
    check(lib.vb_rollout_update(_ptr(window), T, rows, V_in, _ptr(y_own), _ptr(y_halo), n_own, V_out, _ptr(f), F,
                                _ptr(kind), _ptr(src), stream))


def shard_plan(path, world, rank):
    """The destination partition of a model file for `rank` of `world` (host only, no GPU): ranges,
    halos, send lists and the local CSR graphs (sources in local ids)."""
    import json
    n = lib.vb_shard_plan(os.fsencode(path), world, rank, None, 0)
    if n < 0:
        check(-n)
    buf = ctypes.create_string_buffer(int(n) + 16)
    n = lib.vb_shard_plan(os.fsencode(path), world, rank, buf, len(buf))
    if n < 0:
        check(-n)
    return json.loads(buf.value.decode())


def nccl_unique_id():
    b = ctypes.create_string_buffer(128)
    check(lib.vb_nccl_unique_id(b))
    return bytes(b.raw)


def launch_count():
    return int(lib.vb_launch_count())


def check_device():
    check(lib.vb_check_device())


class Tiles:
    """Destination tiles of a CSR graph for the shared-memory-staged fp16 attention (vb_tiles_*)."""

    SMEM, TC = 0, 1  # kind: CUDA-core shared-memory tiles, or the tile-sparse tensor-core kernel's tiles

    def __init__(self, row_ptr, src, attr_csr, n_src, head_dim, kind=0):
        rp = np.ascontiguousarray(row_ptr, np.int32)
        s = np.ascontiguousarray(src, np.int32)
        at = np.ascontiguousarray(attr_csr, np.float32)
        h = ctypes.c_void_p()
        check(lib.vb_tiles_create_kind(_ptr(rp), _ptr(s), _ptr(at), at.shape[1], n_src, len(rp) - 1, head_dim, kind,
                                       ctypes.byref(h)))
        self._h = h

    def attention(self, dst_lo, n_rows, q, ldq, k, v, ldkv, xr, ldxr, out, ldo, w_e, C, heads, head_dim, stream=None):
        check(lib.vb_attention_tiled(self._h, dst_lo, n_rows, _ptr(q), ldq, _ptr(k), _ptr(v), ldkv, _ptr(xr), ldxr,
                                     _ptr(out), ldo, _ptr(w_e), C, heads, head_dim, stream))

    def __del__(self):
        try:
            if self._h:
                lib.vb_tiles_free(self._h)
        except Exception:
            pass


def tile_plan(row_ptr, src, attr_csr, n_src, kind=0):
    """The host tile plan (vb_tile_plan): dict of tiles [n, 4] {row0, nrows, src0, nsrc}, srcs, heavy rows
    and the packed edge records [E, 4] float32 (slot or source as int bits in column 3)."""
    rp = np.ascontiguousarray(row_ptr, np.int32)
    s = np.ascontiguousarray(src, np.int32)
    at = np.ascontiguousarray(attr_csr, np.float32)
    cnt = np.zeros(3, np.int64)
    args = (_ptr(rp), _ptr(s), _ptr(at), at.shape[1], n_src, len(rp) - 1, kind)
    check(lib.vb_tile_plan(*args, _ptr(cnt), None, None, None, None))
    tiles = np.empty((int(cnt[0]), 4), np.int32)
    srcs = np.empty(int(cnt[1]), np.int32)
    heavy = np.empty(int(cnt[2]), np.int32)
    edges = np.empty((len(s), 4), np.float32)
    check(lib.vb_tile_plan(*args, _ptr(cnt), _ptr(tiles), _ptr(srcs), _ptr(heavy), _ptr(edges)))
    return {"tiles": tiles, "srcs": srcs, "heavy": heavy, "edges": edges}


def _bind_tiles(L):
    P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    L.vb_tiles_create.argtypes = [P, P, P, I, I64, I64, I, P]
    L.vb_tiles_create.restype = I
    L.vb_tiles_create_kind.argtypes = [P, P, P, I, I64, I64, I, I, P]
    L.vb_tile_plan.argtypes = [P, P, P, I, I64, I64, I, P, P, P, P, P]
    L.vb_tile_plan.restype = I
    L.vb_tiles_create_kind.restype = I
    L.vb_attention_tiled.argtypes = [P, I64, I64, P, I64, P, P, I64, P, I64, P, I64, P, I, I, I, P]
    L.vb_attention_tiled.restype = I
    L.vb_tiles_free.argtypes = [P]
    L.vb_tiles_free.restype = None
