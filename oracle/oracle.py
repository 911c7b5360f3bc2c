"""ctypes wrapper of the CPU oracle (liboracle.so). TEST INFRASTRUCTURE ONLY:
imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
never by the product library. See forge_oracle.h for the reference lines
each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libcpu_ref.so")

OR_MAT_F32, OR_MAT_BF16, OR_MAT_Q4 = 0, 1, 2
OR_KV_BF16, OR_ACT_BF16, OR_NO_ROPE = 1, 2, 4


class OrMat(C.Structure):
    _fields_ = [("kind", C.c_int32), ("group", C.c_int32), ("rows", C.c_int64), ("cols", C.c_int64),
                ("w", C.c_void_p), ("scales", C.c_void_p)]


class OrLayer(C.Structure):
    _fields_ = [("g1", C.c_void_p), ("wq", OrMat), ("wk", OrMat), ("wv", OrMat), ("wo", OrMat),
                ("g2", C.c_void_p), ("wg", OrMat), ("wu", OrMat), ("wd", OrMat)]


class OrModel(C.Structure):
    _fields_ = [("n_layer", C.c_int32), ("d", C.c_int32), ("n_head", C.c_int32), ("n_kv", C.c_int32),
                ("hd", C.c_int32), ("ffn", C.c_int32), ("vocab", C.c_int32), ("eps", C.c_float),
                ("theta", C.c_float), ("layers", C.POINTER(OrLayer)), ("emb", OrMat),
                ("gF", C.c_void_p), ("head", OrMat)]


_lib = None


def build() -> None:
    subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, stdout=subprocess.DEVNULL)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int
        sig = {
            "or_f32_to_bf16_n": (None, [vp, vp, i64]),
            "or_bf16_to_f32_n": (None, [vp, vp, i64]),
            "or_flame_fill_lcg": (None, [vp, i64, i64, C.c_double]),
            "or_int4_quant_fwd": (None, [vp, vp, vp, vp, vp, i32, i32]),
            "or_int4_pack": (None, [vp, vp, i32, C.c_double, i32]),
            "or_int4_unpack": (None, [vp, vp, i32, C.c_double, i32]),
            "or_q4g_quantize_bf16": (i32, [vp, i64, i64, i32, vp, vp]),
            "or_q4g_dequant": (i32, [vp, vp, i64, i64, i32, vp]),
            "or_fill_normal_bf16": (None, [vp, i64, C.c_uint64, C.c_uint64, C.c_float]),
            "or_normal_at": (C.c_double, [C.c_uint64, C.c_uint64]),
            "or_rope_table": (None, [vp, vp, i32, i32, C.c_double]),
            "or_decode_step": (i32, [C.POINTER(OrModel), vp, vp, i32, i32, vp, vp, i32, vp, vp, vp]),
            "or_full_forward": (i32, [C.POINTER(OrModel), vp, i32, vp]),
            "or_greedy": (i32, [C.POINTER(OrModel), i32, vp, i32, i32, i32, vp, vp]),
            "or_flash_decode_single": (None, [vp, vp, vp, i32, i32, i32, vp]),
            "or_matmul_f64": (None, [vp, vp, vp, i32, i32, i32]),
            "or_num_threads": (i32, []),
            "or_ref_lcg_f32": (None, [vp, vp, i64]),
            "or_sampler_rand": (C.c_double, [vp]),
            "or_sample_token": (i32, [vp, i32, C.c_double, i32, C.c_double, vp, vp]),
            "or_dt_exp": (C.c_double, [C.c_double]),
            "or_attn_scale": (C.c_double, [i64]),
            "or_train_rmsnorm_rows": (None, [vp, i64, i64, C.c_double, vp]),
            "or_train_rmsnorm_bwd_rows": (None, [vp, vp, i64, i64, vp]),
            "or_train_adamw": (None, [vp, vp, vp, vp, i64] + [C.c_double] * 5 + [i64, vp]),
            "or_train_rope": (None, [vp, vp, vp, i64, i64, i64, i32, vp]),
            "or_train_silu": (None, [vp, vp, i64, i32, vp]),
            "or_train_attn_fwd": (None, [vp, vp, vp, i64, i64, i64, i64, vp, vp]),
            "or_train_attn_bwd": (None, [vp, vp, vp, vp, vp, i64, i64, i64, i64, vp, vp, vp]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


def P(a):
    return a.ctypes.data if a is not None else None


# ---- scalar formats -----------------------------------------------------------
def f32_to_bf16(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_bf16_n(P(x), P(out), x.size)
    return out


def sample_token(logits, temperature, top_k, top_p, state):
    """One draw of the reference sampler; returns (token, new_state, probs)."""
    x = np.ascontiguousarray(logits, np.float32)
    st = C.c_int64(int(state))
    probs = np.zeros(x.size, np.float32)
    tok = lib().or_sample_token(P(x), x.size, float(temperature), int(top_k), float(top_p), C.byref(st), P(probs))
    return tok, st.value, probs


def bf16_to_f32(b):
    b = np.ascontiguousarray(b, np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().or_bf16_to_f32_n(P(b), P(out), b.size)
    return out


def fill_normal_bf16(n, seed, offset, std):
    out = np.empty(n, np.uint16)
    lib().or_fill_normal_bf16(P(out), n, seed, offset, std)
    return out


def q4g_quantize(w_bf16, group=128):
    w = np.ascontiguousarray(w_bf16, np.uint16)
    rows, K = w.shape
    codes = np.empty((rows, K // 2), np.uint8)
    scales = np.empty((rows, K // group), np.uint16)
    assert lib().or_q4g_quantize_bf16(P(w), rows, K, group, P(codes), P(scales)) == 0
    return codes, scales


def q4g_dequant(codes, scales, K, group=128):
    rows = codes.shape[0]
    out = np.empty((rows, K), np.float32)
    assert lib().or_q4g_dequant(P(np.ascontiguousarray(codes)), P(np.ascontiguousarray(scales)),
                                rows, K, group, P(out)) == 0
    return out


def rope_table(lmax, hd, theta=10000.0):
    c = np.empty((lmax, hd // 2), np.float32)
    s = np.empty_like(c)
    lib().or_rope_table(P(c), P(s), lmax, hd, theta)
    return c, s


# ---- synthetic model ----------------------------------------------------------
MAT_NAMES = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


class OracleModel:
    """Weights + ctypes structs for the oracle. Synthetic weights follow the
    device's stream assignment: tensor t uses (seed, t << 40) with emb t=0,
    head t=1 and layer l matrix j at t = 2 + 7*l + j; gains are 1.0."""

    def __init__(self, n_layer, d, n_head, n_kv, hd, ffn, vocab, *, q4=False, tied=False,
                 eps=1e-5, theta=10000.0, seed=1234, std=0.02, weights=None, keep_bf16=True):
        """keep_bf16=False (synthetic int4 models only): each layer matrix is
        generated, quantised and its bf16 copy dropped, so a full-size model
        (7B: 13 GB of bf16) holds only its int4 codes and scales."""
        self.cfg = dict(n_layer=n_layer, d=d, n_head=n_head, n_kv=n_kv, hd=hd, ffn=ffn, vocab=vocab)
        self.q4, self.tied = q4, tied
        shapes = {"wq": (n_head * hd, d), "wk": (n_kv * hd, d), "wv": (n_kv * hd, d),
                  "wo": (d, n_head * hd), "wg": (ffn, d), "wu": (ffn, d), "wd": (d, ffn)}
        self.keep = []
        self.bf16 = {}   # logical bf16 weights (what the device is given)
        lazy = weights is None and q4 and not keep_bf16
        if weights is None:
            self.bf16["emb"] = fill_normal_bf16(vocab * d, seed, 0, std).reshape(vocab, d)
            if not tied:
                self.bf16["head"] = fill_normal_bf16(vocab * d, seed, 1 << 40, std).reshape(vocab, d)
            if not lazy:
                for l in range(n_layer):
                    for j, nm in enumerate(MAT_NAMES):
                        r, c = shapes[nm]
                        self.bf16[(l, nm)] = fill_normal_bf16(r * c, seed, (2 + 7 * l + j) << 40, std).reshape(r, c)
            self.gains = {k: np.ones(d, np.float32) for k in
                          ["gF"] + [(l, g) for l in range(n_layer) for g in ("g1", "g2")]}
        else:
            self.bf16, self.gains = weights
        self.layers = (OrLayer * n_layer)()
        for l in range(n_layer):
            L = self.layers[l]
            L.g1 = P(self._k(self.gains[(l, "g1")]))
            L.g2 = P(self._k(self.gains[(l, "g2")]))
            for j, nm in enumerate(MAT_NAMES):
                if lazy:
                    r, c = shapes[nm]
                    w = fill_normal_bf16(r * c, seed, (2 + 7 * l + j) << 40, std).reshape(r, c)
                    setattr(L, nm, self._mat(w, q4))
                    del w
                else:
                    setattr(L, nm, self._mat(self.bf16[(l, nm)], q4))
        m = OrModel()
        m.n_layer, m.d, m.n_head, m.n_kv, m.hd, m.ffn, m.vocab = n_layer, d, n_head, n_kv, hd, ffn, vocab
        m.eps, m.theta = eps, theta
        m.layers = C.cast(self.layers, C.POINTER(OrLayer))
        m.emb = self._mat(self.bf16["emb"], False)
        m.gF = P(self._k(self.gains["gF"]))
        m.head = m.emb if tied else self._mat(self.bf16["head"], False)
        self.m = m

    def _k(self, a):
        self.keep.append(a)
        return a

    def _mat(self, w_bf16, q4):
        rows, cols = w_bf16.shape
        if w_bf16.dtype == np.float32:  # fp32 weights (the reference's own check inputs)
            w = self._k(np.ascontiguousarray(w_bf16))
            return OrMat(OR_MAT_F32, 0, rows, cols, P(w), None)
        if q4:
            codes, scales = q4g_quantize(w_bf16)
            self._k(codes), self._k(scales)
            return OrMat(OR_MAT_Q4, 128, rows, cols, P(codes), P(scales))
        self._k(w_bf16)
        return OrMat(OR_MAT_BF16, 0, rows, cols, P(w_bf16), None)

    def new_cache(self, B, lmax):
        c = self.cfg
        shape = (c["n_layer"], B, c["n_kv"], lmax, c["hd"])
        return np.zeros(shape, np.float32), np.zeros(shape, np.float32)

    def decode_step(self, kc, vc, tok, pos, flags=OR_KV_BF16, want_hidden=False):
        B = len(tok)
        tok = np.ascontiguousarray(tok, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        logits = np.empty((B, self.cfg["vocab"]), np.float32)
        am = np.empty(B, np.int32)
        hid = np.empty((B, self.cfg["d"]), np.float64) if want_hidden else None
        rc = lib().or_decode_step(C.byref(self.m), P(kc), P(vc), kc.shape[3], B, P(tok), P(pos), flags,
                                  P(logits), P(am), P(hid))
        assert rc == 0
        return (logits, am, hid) if want_hidden else (logits, am)

    def full_forward(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.cfg["vocab"], np.float64)
        assert lib().or_full_forward(C.byref(self.m), P(ids), len(ids), P(out)) == 0
        return out

    def greedy(self, prompt, n_gen, flags=OR_KV_BF16):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n_gen, np.int32)
        margins = np.empty(n_gen, np.float32)
        lmax = len(prompt) + n_gen
        assert lib().or_greedy(C.byref(self.m), lmax, P(prompt), len(prompt), n_gen, flags, P(out), P(margins)) == 0
        return out, margins


# ---- the reference's own single-layer decode (tool/decode_eager_baseline.cu) ---
REF_D, REF_NH, REF_HD, REF_FF = 768, 12, 64, 3072  # its fixed #defines (:42-45)


def ref_inputs(L):
    """The inputs of the reference's single-layer decode check at cache length
    L, drawn from its LCG in the order of its main()
    (tool/decode_eager_baseline.cu:209-219); fp32 arrays."""
    D, FF = REF_D, REF_FF
    st = np.array([0x12345678], np.uint32)

    def draw(n):
        out = np.empty(n, np.float32)
        lib().or_ref_lcg_f32(P(st), P(out), n)
        return out
    wq = np.float32(0.036)
    a = draw(3 * D).reshape(D, 3)
    x = a[:, 0].copy()
    g1 = np.float32(1) + np.float32(0.1) * a[:, 1]
    g2 = np.float32(1) + np.float32(0.1) * a[:, 2]
    b = draw(4 * D * D).reshape(D * D, 4) * wq
    Wq, Wk, Wv, Wo = (b[:, i].reshape(D, D).copy() for i in range(4))
    c = draw(2 * FF * D).reshape(FF * D, 2) * wq
    Wg, Wu = (c[:, i].reshape(FF, D).copy() for i in range(2))
    Wd = (draw(D * FF) * np.float32(0.018)).reshape(D, FF)
    kv = draw(2 * L * D).reshape(L * D, 2)
    Kc = (kv[:, 0] * wq * np.float32(0.5)).reshape(L, D)
    Vc = kv[:, 1].reshape(L, D).copy()
    return dict(x=x, g1=g1, g2=g2, Wq=Wq, Wk=Wk, Wv=Wv, Wo=Wo, Wg=Wg, Wu=Wu, Wd=Wd, Kc=Kc, Vc=Vc)


def ref_layer_via_oracle(inp, L, flags=OR_NO_ROPE):
    """The oracle's decode step at the reference check's shape: one MHA layer
    (12 heads x 64), fp32 weights, fp32 cache with L rows, no RoPE, eps 1e-5;
    the input row is supplied as a one-row embedding table. Returns the
    layer's output hidden state (f64, [768])."""
    D, NH, HD, FF = REF_D, REF_NH, REF_HD, REF_FF
    w = {(0, "wq"): inp["Wq"], (0, "wk"): inp["Wk"], (0, "wv"): inp["Wv"], (0, "wo"): inp["Wo"],
         (0, "wg"): inp["Wg"], (0, "wu"): inp["Wu"], (0, "wd"): inp["Wd"],
         "emb": inp["x"].reshape(1, D).astype(np.float32)}
    gains = {(0, "g1"): inp["g1"].astype(np.float32), (0, "g2"): inp["g2"].astype(np.float32),
             "gF": np.ones(D, np.float32)}
    m = OracleModel(1, D, NH, NH, HD, FF, 1, tied=True, eps=1e-5, weights=(w, gains))
    kc, vc = m.new_cache(1, L + 1)
    kc[0, 0, :, :L, :] = inp["Kc"].reshape(L, NH, HD).transpose(1, 0, 2)
    vc[0, 0, :, :L, :] = inp["Vc"].reshape(L, NH, HD).transpose(1, 0, 2)
    _, _, hid = m.decode_step(kc, vc, [0], [L], flags=flags, want_hidden=True)
    return hid[0]
def ref_lib():
    """libcpu_ref.so built by oracle/Makefile from the reference source, or None."""
    if not os.path.exists(REF_LIB):
        return None
    L = C.CDLL(REF_LIB)
    vp = C.c_void_p
    L.ref_make_inputs.argtypes = [C.c_int] + [vp] * 12
    L.ref_cpu_ref.argtypes = [vp] * 12 + [C.c_int, vp]
    L.ref_dims.argtypes = [C.POINTER(C.c_int)] * 4
    return L
