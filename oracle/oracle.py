"""ctypes front-end for the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline arm of bench.py as the checker.  The product library never
imports this module.

Each wrapper names the reference function it restates (paths relative to the
rogu3bear/adapter-os tree); the restatement itself is in aos_oracle.cpp.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

MOD_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
NUM_MODS = 7


class OracleRing(C.Structure):
    """40-byte RouterRing device layout (kernel-mtl/src/ring_buffer.rs:44-58)."""

    _fields_ = [
        ("top_k", C.c_uint32),
        ("position", C.c_uint32),
        ("indices", C.c_uint16 * 8),
        ("gates_q15", C.c_int16 * 8),
    ]


RING_DTYPE = np.dtype(
    [("top_k", "<u4"), ("position", "<u4"), ("indices", "<u2", (8,)), ("gates_q15", "<i2", (8,))]
)
assert RING_DTYPE.itemsize == 40


class OracleModel(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32), ("inter", C.c_uint32), ("vocab", C.c_uint32),
        ("n_layers", C.c_uint32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("rope_mlx_as_written", C.c_uint32),
        ("embed", C.c_void_p), ("lm_head", C.c_void_p), ("final_norm", C.c_void_p),
        ("attn_norm", C.c_void_p), ("mlp_norm", C.c_void_p),
        ("w", C.c_void_p * NUM_MODS),
    ]


class OracleAdapters(C.Structure):
    _fields_ = [
        ("n_adapters", C.c_uint32), ("rank", C.c_void_p), ("alpha", C.c_void_p),
        ("A", C.c_void_p), ("B", C.c_void_p),
    ]


class OracleKV(C.Structure):
    _fields_ = [
        ("k_pool", C.c_void_p), ("v_pool", C.c_void_p),
        ("num_blocks", C.c_uint32), ("block_size", C.c_uint32), ("max_blocks", C.c_uint32),
        ("block_tables", C.c_void_p), ("ctx_lens", C.c_void_p),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc, no CUDA)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.oracle_quantize_gate.restype = C.c_int16
        L.oracle_quantize_gate.argtypes = [C.c_float]
        L.oracle_deterministic_softmax.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_void_p]
        L.oracle_route_batch.argtypes = [
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
            C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p,
            C.c_void_p, C.c_int,
        ]
        L.oracle_lora_op_f32.argtypes = [
            C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
            C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
        ]
        L.oracle_liquid_blend_f32.argtypes = [
            C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
        ]
        L.oracle_layer_step.argtypes = [
            C.POINTER(OracleModel), C.POINTER(OracleAdapters), C.c_uint32, C.c_void_p,
            C.c_uint32, C.POINTER(OracleKV), C.c_void_p, C.c_int, C.c_int,
        ]
        L.oracle_decode_step.argtypes = [
            C.POINTER(OracleModel), C.POINTER(OracleAdapters), C.c_void_p, C.c_void_p,
            C.c_uint32, C.POINTER(OracleKV), C.c_uint32, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
        ]
        L.oracle_rope_table.argtypes = [C.c_uint32, C.c_float, C.c_uint32, C.c_uint32, C.c_void_p]
        L.oracle_bf16_to_f32.restype = C.c_float
        L.oracle_bf16_to_f32.argtypes = [C.c_uint16]
        L.oracle_blake3.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        L.oracle_blake3_incremental.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        L.oracle_aos_validate.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        L.oracle_greedy.restype = C.c_uint32
        L.oracle_greedy.argtypes = [C.c_void_p, C.c_uint32]
        L.oracle_sample.restype = C.c_uint32
        L.oracle_sample.argtypes = [C.c_void_p, C.c_uint32, C.c_float, C.c_int, C.c_uint32, C.c_int, C.c_float,
                                    C.c_float]
        L.oracle_f32_to_bf16.restype = C.c_uint16
        L.oracle_f32_to_bf16.argtypes = [C.c_float]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------------ router
def blake3(data: bytes, incremental=False) -> bytes:
    """BLAKE3 digest (B3Hash::hash, adapteros-infra-common/src/hash.rs:22-27;
    the `blake3` crate 1.8.3 restated in aos_archive_oracle.cpp)."""
    buf = C.create_string_buffer(bytes(data), max(1, len(data)))
    out = C.create_string_buffer(32)
    (lib().oracle_blake3_incremental if incremental else lib().oracle_blake3)(buf, len(data), out)
    return out.raw


AOS_RULES = {0: "ok", 1: "too small", 2: "bad magic", 3: "index offset", 4: "reserved bytes", 5: "no index flag",
             6: "index beyond file", 7: "index size", 8: "manifest beyond file", 9: "manifest overlaps index",
             10: "backend tag", 11: "segment overlaps index", 12: "segment overlaps manifest",
             13: "segment beyond file", 14: "segment hash"}


def aos_validate(data: bytes):
    """open_aos (adapteros-aos/src/writer.rs:407-558): (rule code, n_segments)."""
    buf = C.create_string_buffer(bytes(data), max(1, len(data)))
    n = C.c_uint32(0)
    rc = lib().oracle_aos_validate(buf, len(data), C.byref(n))
    return int(rc), int(n.value)


def sample(logits, u=None, temperature=1.0, top_k=None, top_p=None, greedy=False):
    """Generator::next_token / greedy (lora-worker/src/generation.rs:321-490)
    per row of logits [T, V] f32; u [T] uniform draws.  Returns uint32 [T]."""
    x = np.ascontiguousarray(logits, np.float32)
    if x.ndim == 1:
        x = x[None]
    T, V = x.shape
    out = np.zeros(T, np.uint32)
    for t in range(T):
        row = x[t]
        if greedy:
            out[t] = lib().oracle_greedy(_p(row), V)
        else:
            out[t] = lib().oracle_sample(_p(row), V, float(temperature), int(top_k is not None),
                                         int(top_k or 0), int(top_p is not None), float(top_p or 0.0),
                                         float(u[t]))
    return out


def quantize_gate(g: float) -> int:
    """quantization.rs:172-175."""
    return int(lib().oracle_quantize_gate(float(g)))


def deterministic_softmax(scores, tau: float) -> np.ndarray:
    """router.rs:1340-1411."""
    s = np.ascontiguousarray(scores, dtype=np.float32)
    out = np.zeros(len(s), dtype=np.float32)
    lib().oracle_deterministic_softmax(_p(s), len(s), float(tau), _p(out))
    return out


def route_batch(priors, stable_ids=None, k=4, tau=1.0, eps=0.02, routing_bias=1.0,
                version_weights=None, allowed=None, positions=None, n_threads=0):
    """Route each row of ``priors`` [T, N] with the reference router
    (router.rs:1567-1952).  Returns (rings structured array [T], entropy [T],
    status [T], overall status)."""
    pr = np.ascontiguousarray(priors, dtype=np.float32)
    if pr.ndim == 1:
        pr = pr[None, :]
    T, N = pr.shape
    sid = np.ascontiguousarray(
        np.arange(N, dtype=np.uint64) if stable_ids is None else stable_ids, dtype=np.uint64)
    vw = None if version_weights is None else np.ascontiguousarray(version_weights, dtype=np.float32)
    al = None if allowed is None else np.ascontiguousarray(allowed, dtype=np.uint8)
    pos = None if positions is None else np.ascontiguousarray(positions, dtype=np.uint32)
    rings = np.zeros(T, dtype=RING_DTYPE)
    ent = np.zeros(T, dtype=np.float32)
    st = np.zeros(T, dtype=np.int32)
    rc = lib().oracle_route_batch(_p(pr), _p(sid), _p(vw), _p(al), T, N, int(k), float(tau),
                                  float(eps), float(routing_bias), _p(pos), _p(rings), _p(ent),
                                  _p(st), int(n_threads))
    return rings, ent, st, rc


# ------------------------------------------------------------------ fp32 LoRA op
def lora_op_f32(x, W, A, B, rings, alpha=None, n_threads=0):
    """cpu_lora_forward + liquid blend loop (kernel_testing.rs:220-257, liquid.rs:222-250)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    rings = np.ascontiguousarray(rings, dtype=RING_DTYPE)
    T, ind = x.shape
    outd = W.shape[0]
    n_ad, rank, _ = A.shape
    al = None if alpha is None else np.ascontiguousarray(alpha, dtype=np.float32)
    y = np.zeros((T, outd), dtype=np.float32)
    rc = lib().oracle_lora_op_f32(_p(x), T, ind, outd, _p(W), _p(A), _p(B), n_ad, rank, _p(al),
                                  _p(rings), _p(y), int(n_threads))
    if rc != 0:
        raise RuntimeError(f"oracle_lora_op_f32 failed: {rc}")
    return y


def liquid_blend_f32(x, As, Bs, alphas, coeffs, out_dim):
    """blend_and_forward_reference (liquid.rs:163-251). As[i]: [rank, in], Bs[i]: [rows, rank]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    As = [np.ascontiguousarray(a, dtype=np.float32) for a in As]
    Bs = [np.ascontiguousarray(b, dtype=np.float32) for b in Bs]
    n = len(As)
    pa = (C.c_void_p * max(1, n))(*[_p(a) for a in As])
    pb = (C.c_void_p * max(1, n))(*[_p(b) for b in Bs])
    rank = np.array([a.shape[0] for a in As], dtype=np.uint32)
    rows = np.array([b.shape[0] for b in Bs], dtype=np.uint32)
    al = np.ascontiguousarray(alphas, dtype=np.float32)
    co = np.ascontiguousarray(coeffs, dtype=np.float32)
    y = np.zeros(out_dim, dtype=np.float32)
    rc = lib().oracle_liquid_blend_f32(_p(x), len(x), out_dim, n, C.cast(pa, C.c_void_p),
                                       C.cast(pb, C.c_void_p), _p(rank), _p(rows), _p(al), _p(co), _p(y))
    return y, rc


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    finite = np.isfinite(a)
    if finite.all():
        # |x| < inf: adding at most 0x8000 cannot carry out of 32 bits
        return ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    r = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    r[~finite] = (u[~finite] >> 16).astype(np.uint16)
    nan = np.isnan(a)
    r[nan] |= 0x40
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def rope_table(head_dim, theta, max_pos, mlx_as_written=False):
    t = np.zeros((max_pos, head_dim // 2, 2), dtype=np.float32)
    lib().oracle_rope_table(head_dim, float(theta), int(bool(mlx_as_written)), max_pos, _p(t))
    return t


# ------------------------------------------------------------------ decoder
class HostModel:
    """Host-side bf16 weights of a decoder in the layout both the oracle and
    the CUDA library accept: per layer, per module W [out, in] (uint16 bf16 bits)."""

    def __init__(self, hidden, n_heads, n_kv_heads, head_dim, inter, vocab, n_layers,
                 rms_eps=1e-5, rope_theta=1e6, rope_mlx_as_written=False):
        self.hidden, self.n_heads, self.n_kv_heads = hidden, n_heads, n_kv_heads
        self.head_dim, self.inter, self.vocab, self.n_layers = head_dim, inter, vocab, n_layers
        self.rms_eps, self.rope_theta = rms_eps, rope_theta
        self.rope_mlx_as_written = rope_mlx_as_written
        self.embed = None
        self.lm_head = None
        self.final_norm = None
        self.attn_norm = [None] * n_layers
        self.mlp_norm = [None] * n_layers
        self.w = [[None] * n_layers for _ in range(NUM_MODS)]

    def mod_shape(self, m):
        q = self.n_heads * self.head_dim
        kv = self.n_kv_heads * self.head_dim
        H, I = self.hidden, self.inter
        return [(q, H), (kv, H), (kv, H), (H, q), (I, H), (I, H), (H, I)][m]

    @staticmethod
    def random(rng, hidden, n_heads, n_kv_heads, head_dim, inter, vocab, n_layers, std=0.02,
               with_embed=True, **kw):
        """Seeded random-init weights ~N(0, std) rounded to bf16; norms ~1+N(0,0.1)."""
        m = HostModel(hidden, n_heads, n_kv_heads, head_dim, inter, vocab, n_layers, **kw)

        def rnd(*shape, s=std):
            return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * s)

        if with_embed:
            m.embed = rnd(vocab, hidden, s=1.0)
            m.lm_head = rnd(vocab, hidden)
            m.final_norm = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(hidden, dtype=np.float32))
        for l in range(n_layers):
            m.attn_norm[l] = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(hidden, dtype=np.float32))
            m.mlp_norm[l] = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(hidden, dtype=np.float32))
            for mod in range(NUM_MODS):
                m.w[mod][l] = rnd(*m.mod_shape(mod))
        return m

    def _struct(self):
        keep = []

        def ptr_array(lst):
            arr = (C.c_void_p * len(lst))(*[_p(a) for a in lst])
            keep.append(arr)
            return C.cast(arr, C.c_void_p)

        s = OracleModel()
        s.hidden, s.n_heads, s.n_kv_heads = self.hidden, self.n_heads, self.n_kv_heads
        s.head_dim, s.inter, s.vocab, s.n_layers = self.head_dim, self.inter, self.vocab, self.n_layers
        s.rms_eps, s.rope_theta = self.rms_eps, self.rope_theta
        s.rope_mlx_as_written = int(bool(self.rope_mlx_as_written))
        s.embed, s.lm_head, s.final_norm = _p(self.embed), _p(self.lm_head), _p(self.final_norm)
        s.attn_norm = ptr_array(self.attn_norm)
        s.mlp_norm = ptr_array(self.mlp_norm)
        for mod in range(NUM_MODS):
            s.w[mod] = ptr_array(self.w[mod])
        return s, keep


class HostAdapters:
    """Adapter pool on the host: per adapter rank, alpha, and per (layer,
    module) A [rank, in] / B [out, rank] bf16 bits (None = module absent).
    Shapes follow MLXLoraModule (mlx_cpp_wrapper_real.cpp:1239-1244)."""

    def __init__(self, model: HostModel, ranks, alphas):
        self.model = model
        self.ranks = [int(r) for r in ranks]
        self.alphas = [float(a) for a in alphas]
        self.n = len(self.ranks)
        self.A = [[[None] * NUM_MODS for _ in range(model.n_layers)] for _ in range(self.n)]
        self.B = [[[None] * NUM_MODS for _ in range(model.n_layers)] for _ in range(self.n)]

    @staticmethod
    def random(rng, model: HostModel, ranks, alphas=None, modules=range(NUM_MODS), std=0.02):
        if alphas is None:
            alphas = [2.0 * r for r in ranks]  # default alpha = 2r (kernel-mtl/src/lib.rs:239-251)
        ad = HostAdapters(model, ranks, alphas)
        for a, r in enumerate(ad.ranks):
            for l in range(model.n_layers):
                for mod in modules:
                    out, inn = model.mod_shape(mod)
                    ad.A[a][l][mod] = f32_to_bf16_bits(rng.standard_normal((r, inn), dtype=np.float32) * std)
                    ad.B[a][l][mod] = f32_to_bf16_bits(rng.standard_normal((out, r), dtype=np.float32) * std)
        return ad

    def _struct(self):
        keep = []
        L = self.model.n_layers
        flatA, flatB = [], []
        for a in range(self.n):
            for l in range(L):
                for mod in range(NUM_MODS):
                    flatA.append(self.A[a][l][mod])
                    flatB.append(self.B[a][l][mod])
        rank = np.array(self.ranks, dtype=np.uint32)
        alpha = np.array(self.alphas, dtype=np.float32)
        pa = (C.c_void_p * max(1, len(flatA)))(*[_p(x) for x in flatA])
        pb = (C.c_void_p * max(1, len(flatB)))(*[_p(x) for x in flatB])
        keep += [rank, alpha, pa, pb]
        s = OracleAdapters()
        s.n_adapters = self.n
        s.rank, s.alpha = _p(rank), _p(alpha)
        s.A, s.B = C.cast(pa, C.c_void_p), C.cast(pb, C.c_void_p)
        return s, keep


class HostKV:
    """Paged KV pools [n_layers][num_blocks][n_kv][block][hd] bf16 bits plus
    per-token block tables and cached lengths."""

    def __init__(self, model: HostModel, num_blocks, block_size, block_tables, ctx_lens,
                 k_pool=None, v_pool=None):
        shape = (model.n_layers, num_blocks, model.n_kv_heads, block_size, model.head_dim)
        self.k_pool = np.zeros(shape, np.uint16) if k_pool is None else k_pool
        self.v_pool = np.zeros(shape, np.uint16) if v_pool is None else v_pool
        self.num_blocks, self.block_size = num_blocks, block_size
        self.block_tables = np.array(block_tables, dtype=np.int32, copy=True)
        self.max_blocks = self.block_tables.shape[1]
        self.ctx_lens = np.array(ctx_lens, dtype=np.int32, copy=True)

    def _struct(self):
        s = OracleKV()
        s.k_pool, s.v_pool = _p(self.k_pool), _p(self.v_pool)
        s.num_blocks, s.block_size, s.max_blocks = self.num_blocks, self.block_size, self.max_blocks
        s.block_tables, s.ctx_lens = _p(self.block_tables), _p(self.ctx_lens)
        return s


def kv_rotate_rows(rows, length, shift):
    """kv_cache_rotate (crates/adapteros-lora-kernel-mtl/shaders/kv_cache.metal:
    200-236) on one sequence's rows [positions, n_kv, head_dim] of one layer:
    for seq_idx < length - shift, dst[seq_idx] = src[seq_idx + shift] (every
    head and dimension); rows past the new length are left as they were.
    Returns the new rows and the new length."""
    if shift > length:
        raise ValueError("shift beyond the sequence length")
    new_len = length - shift
    out = np.array(rows, copy=True)
    for seq_idx in range(new_len):  # the shader's grid x, one position at a time
        out[seq_idx] = rows[seq_idx + shift]
    return out, new_len


def layer_step(model: HostModel, adapters, layer, rings, kv: HostKV, hidden, rounding_mode=0,
               n_threads=0):
    """One decoder layer (mlx_cpp_wrapper_real.cpp:3437-3531); updates hidden
    (uint16 bf16 [T, H]) and the KV pools in place."""
    ms, k1 = model._struct()
    if adapters is not None:
        ad, k2 = adapters._struct()
    else:
        ad, k2 = OracleAdapters(), []
    kvs = kv._struct()
    rings = np.ascontiguousarray(rings, dtype=RING_DTYPE)
    T = hidden.shape[0]
    rc = lib().oracle_layer_step(C.byref(ms), C.byref(ad), layer, _p(rings), T, C.byref(kvs),
                                 _p(hidden), rounding_mode, n_threads)
    if rc != 0:
        raise RuntimeError(f"oracle_layer_step failed: {rc}")
    del k1, k2
    return hidden


def decode_step(model: HostModel, adapters, rings, token_ids, kv: HostKV, n_layers_run=None,
                rounding_mode=0, want_logits=True, n_threads=0):
    ms, k1 = model._struct()
    if adapters is not None:
        ad, k2 = adapters._struct()
    else:
        ad, k2 = OracleAdapters(), []
    kvs = kv._struct()
    rings = np.ascontiguousarray(rings, dtype=RING_DTYPE)
    tok = np.ascontiguousarray(token_ids, dtype=np.int32)
    T = len(tok)
    nl = model.n_layers if n_layers_run is None else n_layers_run
    logits = np.zeros((T, model.vocab), np.float32) if want_logits else None
    hid = np.zeros((T, model.hidden), np.uint16)
    rc = lib().oracle_decode_step(C.byref(ms), C.byref(ad), _p(rings), _p(tok), T, C.byref(kvs), nl,
                                  rounding_mode, _p(logits), _p(hid), n_threads)
    if rc != 0:
        raise RuntimeError(f"oracle_decode_step failed: {rc}")
    del k1, k2
    return logits, hid
