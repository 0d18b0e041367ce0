"""CPU fp32 oracle of the reference's GraphTransformer predict_step (varda.cpp).

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
import this module, and only as the checker; the product never does.

The orchestration below restates the reference CPU backend's forward pass,
src/varda/cpu/backend_cpu.cpp:297-537, with its kernels (Linear, LayerNorm, GELU, graph attention,
CSR build) restated in C in varda_oracle.c (built into _build/liboracle.so by the Makefile). The
restatement is pinned by tests/test_oracle.py against the reference's own golden vectors
(python/tests/synthetic.py, models a-h; committed summaries in tests/golden/) and against the
reference CPU backend compiled from its sources (oracle/_ref/ref_dump).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_NP = {"F32": np.float32, "F16": np.float16, "F64": np.float64, "I64": np.int64, "I32": np.int32,
       "U8": np.uint8, "I8": np.int8, "I16": np.int16, "BOOL": np.bool_}


def build():
    """Compile liboracle.so (and, when the reference sources exist, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            subprocess.run(["make", "-s", "-C", _HERE, "oracle"], check=True)
        L = ctypes.CDLL(path)
        P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.vo_build_csr.argtypes = [P, I64, P, I, I64, I64, P, P, P, P, P]
        L.vo_build_csr.restype = I
        L.vo_linear.argtypes = [P, I64, I64, P, P, I64, I64, P, I64]
        L.vo_layer_norm.argtypes = [P, I64, I64, I64, P, P, F, P, I64]
        L.vo_gelu.argtypes = [P, I64, I]
        L.vo_graph_attention.argtypes = [P, P, P, I, I64, I64, P, I64, P, P, I64, P, P, I, I, P, I64]
        L.vo_set_threads.argtypes = [I]
        _LIB = L
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ safetensors (read only)
def read_safetensors(path):
    """Returns ({name: ndarray}, metadata). Arrays are views of a read-only memory map."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + n
    out = {}
    for k, v in hdr.items():
        if k == "__metadata__":
            continue
        a, b = v["data_offsets"]
        out[k] = np.frombuffer(mm, dtype=_NP[v["dtype"]], count=(b - a) // np.dtype(_NP[v["dtype"]]).itemsize,
                               offset=base + a).reshape(v["shape"])
    return out, hdr.get("__metadata__", {})


# ------------------------------------------------------------------ kernels (C)
def build_csr(edge_index, edge_attr, n_src, n_dst):
    """graph.cpp:17-61 -> (row_ptr, src, edge_id, attr) in CSR order."""
    ei = np.ascontiguousarray(edge_index, dtype=np.int64)
    ea = np.ascontiguousarray(edge_attr, dtype=np.float32)
    E, A = ei.shape[1], ea.shape[1]
    rp = np.empty(n_dst + 1, np.int32)
    src = np.empty(E, np.int32)
    eid = np.empty(E, np.int32)
    at = np.empty((E, A), np.float32)
    bad = np.zeros(1, np.int64)
    rc = lib().vo_build_csr(_p(ei), E, _p(ea), A, n_src, n_dst, _p(rp), _p(src), _p(eid), _p(at), _p(bad))
    if rc == -1:
        raise ValueError(f"edge {int(bad[0])} out of range")
    if rc == -2:
        raise ValueError("graph too large for int32 indices")
    return rp, src, eid, at


def linear(x, w, b):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    lib().vo_linear(_p(x), K, M, _p(np.ascontiguousarray(w)), _p(None if b is None else np.ascontiguousarray(b)),
                    N, K, _p(y), N)
    return y


def layer_norm(x, w, b, eps):
    x = np.ascontiguousarray(x, np.float32)
    M, C = x.shape
    y = np.empty_like(x)
    lib().vo_layer_norm(_p(x), C, M, C, _p(np.ascontiguousarray(w)),
                        _p(None if b is None else np.ascontiguousarray(b)), np.float32(eps), _p(y), C)
    return y


def gelu(x, tanh_approx):
    x = np.ascontiguousarray(x, np.float32).copy()
    lib().vo_gelu(_p(x), x.size, int(tanh_approx))
    return x


def graph_attention(csr, d0, nd, q, k, v, edge_wt, edge_b, heads, head_dim):
    rp, src, _, at = csr
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    C = heads * head_dim
    out = np.empty((nd, C), np.float32)
    lib().vo_graph_attention(_p(rp), _p(src), _p(at), at.shape[1], d0, nd, _p(q), q.shape[1], _p(k), _p(v),
                             k.shape[1], _p(np.ascontiguousarray(edge_wt, np.float32)),
                             _p(None if edge_b is None else np.ascontiguousarray(edge_b, np.float32)),
                             heads, head_dim, _p(out), C)
    return out


# ------------------------------------------------------------------ model
class OracleModel:
    """The reference CPU fp32 backend's predict_step (backend_cpu.cpp), restated."""

    def __init__(self, path, threads=0):
        if threads:
            lib().vo_set_threads(threads)
        t, meta = read_safetensors(path)
        if meta.get("varda_format") != "1":
            raise ValueError(f"{path}: unsupported varda_format")
        self.cfg = cfg = json.loads(meta["config"])
        self.t = t
        d = cfg["dims"]
        self.C, self.heads, self.hd = d["num_channels"], d["num_heads"], d["head_dim"]
        self.mlp, self.n_proc = d["mlp_hidden"], d["num_processor_layers"]
        self.T, self.To = d["n_input_steps"], d.get("n_output_steps", 1)
        self.Vi, self.Vo = d["n_input_vars"], d["n_output_vars"]
        self.G, self.H, self.A = d["n_data_nodes"], d["n_hidden_nodes"], d["node_attr_dim"]
        self.eps = np.float32(d["layer_norm_eps"])
        self.tanh = d["gelu_approximate"] == "tanh"
        self.latent_skip = bool(d["latent_skip"])
        self.absent = set(cfg.get("absent", []))
        ix = cfg["indices"]
        mul, add = t["norm.mul"], t["norm.add"]
        self.mul_in, self.add_in = mul[ix["norm_input"]], add[ix["norm_input"]]
        self.mul_out, self.add_out = mul[ix["norm_output"]], add[ix["norm_output"]]
        self.res_in, self.res_out = ix["residual_input"], ix["residual_output"]
        step = cfg["residual"]["step"]
        self.res_step = step + self.T if step < 0 else step
        self.bounding = cfg["bounding"]
        self.csr = {
            "enc": build_csr(t["graph.enc.edge_index"], t["graph.enc.edge_attr"], self.G, self.H),
            "proc": build_csr(t["graph.proc.edge_index"], t["graph.proc.edge_attr"], self.H, self.H),
            "dec": build_csr(t["graph.dec.edge_index"], t["graph.dec.edge_attr"], self.H, self.G),
        }

    def _b(self, name):
        return None if name in self.absent else self.t[name]

    def _lin(self, name, x):
        return linear(x, self.t[name + ".weight"], self._b(name + ".bias"))

    def _ln(self, name, x):
        return layer_norm(x, self.t[name + ".weight"], self._b(name + ".bias"), self.eps)

    def _source_side(self, blk, xs, mapper):
        """backend_cpu.cpp:297-310: LN_src (processor blocks use ln_dst), then k and v."""
        ln = self._ln(blk + (".ln_src" if mapper else ".ln_dst"), xs)
        return self._lin(blk + ".k", ln), self._lin(blk + ".v", ln)

    def _destination_side(self, blk, g, k, v, xd):
        """backend_cpu.cpp:312-365 over all destinations of graph g."""
        ln = self._ln(blk + ".ln_dst", xd)
        q, xr = self._lin(blk + ".q", ln), self._lin(blk + ".self", ln)
        we = self.t[blk + ".edge.weight"]  # [C, A]
        att = graph_attention(self.csr[g], 0, xd.shape[0], q, k, v, np.ascontiguousarray(we.T),
                              self._b(blk + ".edge.bias"), self.heads, self.hd)
        att = att + xr                                   # a + x_r (backend_cpu.cpp:338)
        h = self._lin(blk + ".proj", att) + xd           # proj(...) + xd (:345)
        m = gelu(self._lin(blk + ".mlp1", self._ln(blk + ".ln_mlp", h)), self.tanh)
        return self._lin(blk + ".mlp2", m) + h           # mlp(LN(h)) + h (:362)

    def predict_step(self, x, hook=None):
        """backend_cpu.cpp:461-537. x: (1, T, G, V_in) fp32 -> y (1, T_out, 1, G, V_out) fp32."""
        rep = (lambda k, a: hook(k, np.array(a, np.float32, copy=True))) if hook else (lambda k, a: None)
        T, G, H, Vi, Vo, To = self.T, self.G, self.H, self.Vi, self.Vo, self.To
        x = np.asarray(x, np.float32).reshape(1, T, G, Vi)
        rep("in.x", x)
        xn = (x * self.mul_in).astype(np.float32)        # x * mul, rounded (two fp32 ops, :470-477)
        xn = (xn + self.add_in).astype(np.float32)
        rep("in.x_norm", xn.reshape(1, T, 1, G, Vi))
        x_src = np.concatenate([xn[0, t] for t in range(T)] + [self.t["nodes.data.attr"]], axis=1)
        rep("enc.x_src", x_src)
        rep("enc.x_dst", self.t["nodes.hidden.attr"])
        # encoder (:367-399)
        es = self._lin("enc.emb_src", x_src)
        rep("enc.emb_src", es)
        k, v = self._source_side("enc.block", es, True)
        ed = self._lin("enc.emb_dst", self.t["nodes.hidden.attr"])
        rep("enc.emb_dst", ed)
        z = self._destination_side("enc.block", "enc", k, v, ed)
        rep("enc.out", z)
        # processor (:401-421)
        h = z
        for i in range(self.n_proc):
            k, v = self._source_side(f"proc.{i}", h, False)
            h = self._destination_side(f"proc.{i}", "proc", k, v, h)
            rep(f"proc.{i}.out", h)
        latent = (h + z).astype(np.float32) if self.latent_skip else h
        rep("latent", latent)
        # decoder (:423-459): source = latent (not embedded), destination = dec.emb_dst(x_src)
        k, v = self._source_side("dec.block", latent, True)
        dd = self._lin("dec.emb_dst", x_src)
        rep("dec.emb_dst", dd)
        bo = self._destination_side("dec.block", "dec", k, v, dd)
        rep("dec.block_out", bo)
        dec = self._lin("dec.out_proj", self._ln("dec.out_norm", bo))
        rep("dec.out", dec)
        # residual on every output step (:504-516)
        y = dec.reshape(G, To, Vo).transpose(1, 0, 2).copy()
        xs = xn[0, self.res_step]
        for ri, ro in zip(self.res_in, self.res_out):
            y[:, :, ro] = y[:, :, ro] + xs[:, ri]
        rep("out.pre_bound", y.reshape(1, To, 1, G, Vo))
        # bounding in config order (:111-136, :521)
        for b in self.bounding:
            idx = b["index"]
            if b["type"] == "relu":
                cur = y[:, :, idx]
                y[:, :, idx] = np.where((cur > 0) | np.isnan(cur), cur, np.float32(0))
                continue
            y[:, :, idx] = np.minimum(np.maximum(y[:, :, idx], np.float32(b["min"])), np.float32(b["max"]))
            if b["type"] == "fraction":
                tot = b["total_index"]
                tsel = [tot[0]] * len(idx) if len(tot) == 1 else tot
                prod = y[:, :, idx] * y[:, :, tsel]
                y[:, :, idx] = prod
        rep("out.norm", y.reshape(1, To, 1, G, Vo))
        y = ((y - self.add_out).astype(np.float32) / self.mul_out).astype(np.float32)   # (:525-530)
        y = y.reshape(1, To, 1, G, Vo)
        rep("out.y", y)
        return y


class StateUpdate:
    """The reference's rollout state update, restated (src/varda/rollout.cpp:28-92, rollout.h:44-64).

    kind[c]: 0 constant (kept), 1 prognostic (from output src[c]), 2 dynamic forcing (column src[c]).
    oldest=False: constants keep the newest slot's own value (ConstantSource::Newest, the default);
    True: they take the oldest slot's old value (ConstantSource::Oldest)."""

    def __init__(self, T, G, V_in, V_out, prog_in, prog_out, dyn_in, const_in, oldest=False):
        def require(ok, what):
            if not ok:
                raise ValueError("rollout: " + what)
        require(T >= 1 and G >= 0 and V_in > 0 and V_out > 0, "bad sizes")
        require(len(prog_in) == len(prog_out), "residual_input and residual_output differ in length")
        self.T, self.G, self.V_in, self.V_out, self.F, self.oldest = T, G, V_in, V_out, len(dyn_in), bool(oldest)
        self.kind = np.full(V_in, -1, np.int8)
        self.src = np.full(V_in, -1, np.int32)

        def claim(c, k, s, what):
            require(0 <= c < V_in, f"{what} index {c} out of range")
            require(self.kind[c] < 0, f"input channel {c} is listed twice ({what})")
            self.kind[c], self.src[c] = k, s
        for i, o in zip(prog_in, prog_out):
            require(0 <= o < V_out, "residual_output index out of range")
            claim(i, 1, o, "prognostic")
        for k, c in enumerate(dyn_in):
            claim(c, 2, k, "dynamic forcing")
        for c in const_in:
            claim(c, 0, -1, "constant forcing")
        for c in range(V_in):
            require(self.kind[c] >= 0, f"input channel {c} is neither prognostic, dynamic forcing nor constant")

    @staticmethod
    def from_config(cfg, oldest=False):
        """StateUpdate::from_config (rollout.cpp:62-68)."""
        if "forcings" not in cfg:
            raise ValueError("rollout: the model config has no `forcings` section")
        d, ix, f = cfg["dims"], cfg["indices"], cfg["forcings"]
        return StateUpdate(d["n_input_steps"], d["n_data_nodes"], d["n_input_vars"], d["n_output_vars"],
                           ix["residual_input"], ix["residual_output"], f["dynamic_input_index"],
                           f["constant_input_index"], oldest)

    def apply(self, w, y, f):
        """StateUpdate::apply (rollout.cpp:70-92) on w (T, G, V_in) in place; y (G, V_out); f (G, F).
        Slot t <- slot t+1 in ascending order, then the newest slot's prognostic and forcing channels;
        constants stay (newest) or take the old oldest slot's value (oldest). Pure copies."""
        if self.F and f is None:
            raise ValueError("rollout: forcings missing")
        oldest = w[0].copy()
        for t in range(self.T - 1):
            w[t] = w[t + 1]
        nw = w[self.T - 1]
        p = np.nonzero(self.kind == 1)[0]
        nw[:, p] = y[:, self.src[p]]
        k = np.nonzero(self.kind == 2)[0]
        if len(k):
            nw[:, k] = f[:, self.src[k]]
        if self.oldest:
            c = np.nonzero(self.kind == 0)[0]
            nw[:, c] = oldest[:, c]


def rollout(model, x0, n_steps, forcings=None, oldest=False):
    """Rollout::run (rollout.cpp:116-155) with replayed forcings (n_steps - 1, G, F): predict, then
    (unless last) the update with forcing s. `model` has predict_step(x) -> (1, 1, 1, G, V_out).
    Returns y (n_steps, G, V_out)."""
    u = StateUpdate.from_config(model.cfg, oldest)
    w = np.array(x0, np.float32, copy=True).reshape(u.T, u.G, u.V_in)
    ys = np.empty((n_steps, u.G, u.V_out), np.float32)
    for s in range(n_steps):
        ys[s] = np.asarray(model.predict_step(w[None])).reshape(u.G, u.V_out)
        if s + 1 < n_steps:
            u.apply(w, ys[s], None if forcings is None else forcings[s])
    return ys


def rel_absmax(a, r):
    """The reference's parity metric (apps/common.h:109-127): max|a-r| / max|r| in float64;
    NaN in a -> inf."""
    a = np.asarray(a, np.float64).ravel()
    r = np.asarray(r, np.float64).ravel()
    if np.isnan(a).any():
        return float("inf")
    mx = np.abs(a - r).max() if a.size else 0.0
    am = np.abs(r).max() if r.size else 0.0
    if am > 0:
        return float(mx / am)
    return float("inf") if mx > 0 else 0.0
