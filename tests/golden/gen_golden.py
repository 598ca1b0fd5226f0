"""Generate tests/golden/*.npz: golden vectors from a pure-Python restatement of the
QwenQwen3.js CPU path, written independently of oracle/qq3_oracle.c.

Why: the reference is JavaScript with no tests, fixtures or golden vectors, and no JS
runtime exists on this machine (nor on the GPU box), so the reference cannot produce
vectors itself.  This script transcribes the JS a second time, as plainly as possible
(Python floats are IEEE doubles like JS numbers; `f32()` marks each Float32Array store),
on micro-sized seeded inputs.  tests/test_oracle.py requires the C oracle to reproduce
these vectors, and the GPU tests compare against the C oracle.  Parity with the reference
itself stays unpinned.

Run:  python tests/golden/gen_golden.py   (rewrites the .npz files in this folder; with the
      argument `kquants`, `qwen3moe` or `qwen3kq`, only that file)
"""
from __future__ import annotations

import math
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))


def f32(v: float) -> float:
    """Store into a Float32Array (round to nearest float)."""
    return float(np.float32(v))


def read_f16(b: bytes, off: int) -> float:
    """DataView.getFloat16(off, true) (tensor.js:21-23)."""
    return float(np.frombuffer(b[off:off + 2], dtype="<f2")[0])


def i8(b: bytes, off: int) -> int:
    return struct.unpack_from("b", b, off)[0]


def matmul_q80(w: bytes, in_dim: int, out_dim: int, x: list) -> list:
    """matmulQ80xF32 (tensor.js:26-53)."""
    bpc = -(-in_dim // 32)
    out = []
    for c in range(out_dim):
        dot = 0.0
        col = c * bpc * 34
        for b in range(bpc):
            bp = col + b * 34
            d = read_f16(w, bp)
            for i in range(32):
                if b * 32 + i >= in_dim:
                    break
                dot += x[b * 32 + i] * i8(w, bp + 2 + i) * d
        out.append(f32(dot))
    return out


def embedding_q80(w: bytes, dim: int, token: int) -> list:
    """embeddingLookupQ80 (tensor.js:56-77)."""
    bpc = -(-dim // 32)
    out = [0.0] * dim
    col = token * bpc * 34
    for b in range(bpc):
        bp = col + b * 34
        d = read_f16(w, bp)
        for i in range(32):
            if b * 32 + i < dim:
                out[b * 32 + i] = f32(i8(w, bp + 2 + i) * d)
    return out


def rmsnorm(x: list, w: list, eps: float) -> list:
    """rmsnorm (tensor.js:103-114)."""
    s = 0.0
    for v in x:
        s += v * v
    inv = 1.0 / math.sqrt(s / len(x) + eps)
    return [f32(w[i] * x[i] * inv) for i in range(len(x))]


def per_head_rmsnorm(x: list, nh: int, hd: int, w: list, eps: float) -> list:
    out = []
    for h in range(nh):
        out += rmsnorm(x[h * hd:(h + 1) * hd], w, eps)
    return out


def rope(x: list, nh: int, hd: int, pos: int, base: float) -> list:
    """applyRoPE (tensor.js:132-147)."""
    x = list(x)
    half = hd >> 1
    for h in range(nh):
        o = h * hd
        for i in range(half):
            freq = 1.0 / math.pow(base, i / half)
            th = pos * freq
            c, s = math.cos(th), math.sin(th)
            x0, x1 = x[o + i], x[o + i + half]
            x[o + i] = f32(x0 * c - x1 * s)
            x[o + i + half] = f32(x0 * s + x1 * c)
    return x


def softmax(a: list) -> list:
    """softmaxInPlace (tensor.js:150-164)."""
    a = list(a)
    mx = a[0]
    for v in a[1:]:
        if v > mx:
            mx = v
    s = 0.0
    for i in range(len(a)):
        a[i] = f32(math.exp(a[i] - mx))
        s += a[i]
    inv = 1.0 / s
    return [f32(v * inv) for v in a]


def silu(a):
    return [f32(v * (1.0 / (1.0 + math.exp(-v)))) for v in a]


def mul(a, b):
    return [f32(a[i] * b[i]) for i in range(len(a))]


def add(a, b):
    return [f32(a[i] + b[i]) for i in range(len(a))]


def argmax_first(a) -> int:
    m = 0
    for i in range(1, len(a)):
        if a[i] > a[m]:
            m = i
    return m


class Weights:
    def __init__(self, tensors):
        self.t = tensors  # name -> (type, ne, raw uint8)

    def has(self, n):
        return n in self.t

    def raw(self, n) -> bytes:
        return self.t[n][2].tobytes()

    def ne(self, n):
        return self.t[n][1]

    def f32v(self, n) -> list:
        return [float(v) for v in self.t[n][2].view(np.float32)]

    def mm(self, n, x, expert=None):
        ne = self.ne(n)
        raw = self.raw(n)
        if self.t[n][0] in KQ_BYTES:  # matmulGeneric's k-quant cases (tensor.js:485-496)
            return matmul_kq(self.t[n][0], raw, ne[0], ne[1], x)
        if expert is not None:
            bpc = -(-ne[0] // 32) * 34
            raw = raw[expert * ne[1] * bpc:(expert + 1) * ne[1] * bpc]  # _expertSlice (lfm2-engine.js:490-505)
        return matmul_q80(raw, ne[0], ne[1], x)


class Engine:
    """Qwen3Engine.forward / Lfm2Engine.forward for micro models."""

    def __init__(self, W: Weights, cfg: dict):
        self.W, self.c = W, cfg
        self.kv = {}
        self.conv = {}
        self.mask = set()

    def attention(self, l, normed, pos, slot):
        c, W = self.c, self.W
        b = f"blk.{l}."
        nh, nkv, hd, eps = c["n_head"], c["n_head_kv"], c["head_dim"], c["eps"]
        q = per_head_rmsnorm(W.mm(b + "attn_q.weight", normed), nh, hd, W.f32v(b + "attn_q_norm.weight"), eps)
        k = per_head_rmsnorm(W.mm(b + "attn_k.weight", normed), nkv, hd, W.f32v(b + "attn_k_norm.weight"), eps)
        v = W.mm(b + "attn_v.weight", normed)
        q = rope(q, nh, hd, pos, c["rope"])
        k = rope(k, nkv, hd, pos, c["rope"])
        self.kv[(slot, pos)] = (k, v)  # KVCache.store
        scale = 1.0 / math.sqrt(hd)
        out = [0.0] * (nh * hd)
        for h in range(nh):
            kvh = int(h * nkv / nh)
            sc = []
            for p in range(pos + 1):
                kk = self.kv[(slot, p)][0][kvh * hd:(kvh + 1) * hd]
                dot = 0.0
                for d in range(hd):
                    dot += q[h * hd + d] * kk[d]
                sc.append(f32(dot * scale))
            sc = softmax(sc)
            for p in range(pos + 1):
                w = sc[p]
                if w == 0:
                    continue
                vv = self.kv[(slot, p)][1][kvh * hd:(kvh + 1) * hd]
                for d in range(hd):
                    out[h * hd + d] = f32(out[h * hd + d] + vv[d] * w)
        return W.mm(b + "attn_output.weight", out)

    def shortconv(self, l, normed):
        """Lfm2Engine._shortConv (lfm2-engine.js:282-325)."""
        W, E = self.W, self.c["n_embd"]
        b = f"blk.{l}."
        bcx = W.mm(b + "shortconv.in_proj.weight", normed)
        bx = [f32(bcx[d] * bcx[2 * E + d]) for d in range(E)]
        kern = W.f32v(b + "shortconv.conv.weight")
        st = self.conv.setdefault(l, [[0.0] * E, [0.0] * E])
        co = [f32(kern[d * 3] * st[0][d] + kern[d * 3 + 1] * st[1][d] + kern[d * 3 + 2] * bx[d]) for d in range(E)]
        self.conv[l] = [st[1], bx]
        y = [f32(bcx[E + d] * co[d]) for d in range(E)]
        return W.mm(b + "shortconv.out_proj.weight", y)

    def moe_qwen3(self, l, normed):
        """Qwen3Engine._moEFFN (qwen3-engine.js:304-362): softmax router, stable top-k, weights
        renormalised by their plain sum. Returns (out, record)."""
        W, c = self.W, self.c
        b = f"blk.{l}."
        ne, k = c["n_expert"], c["n_used"]
        probs = softmax(W.mm(b + "ffn_gate_inp.weight", normed))
        top = sorted(range(ne), key=lambda e: -probs[e])[:k]  # stable sort, descending
        tw = [probs[e] for e in top]
        s = 0.0
        for w in tw:
            s += w
        inv = 1.0 / s if s > 0 else 0.0
        rec = [float(e) for e in top] + [f32(w * inv) for w in tw] + probs
        out = [0.0] * c["n_embd"]
        for j, e in enumerate(top):
            if e in self.mask:
                continue
            weight = tw[j] * inv
            g = silu(W.mm(b + "ffn_gate_exps.weight", normed, e))
            g = mul(g, W.mm(b + "ffn_up_exps.weight", normed, e))
            dn = W.mm(b + "ffn_down_exps.weight", g, e)
            out = [f32(out[i] + weight * dn[i]) for i in range(len(out))]
        return out, rec

    def moe(self, l, normed):
        """Lfm2Engine._moEFFN (lfm2-engine.js:413-487). Returns (out, record)."""
        W, c = self.W, self.c
        if c["arch"] == "qwen3moe":
            return self.moe_qwen3(l, normed)
        b = f"blk.{l}."
        ne, k = c["n_expert"], c["n_used"]
        logits = W.mm(b + "ffn_gate_inp.weight", normed)
        rw = [f32(1.0 / (1.0 + math.exp(-v))) for v in logits]
        sel = list(rw)
        if W.has(b + "exp_probs_b.bias"):
            bias = W.f32v(b + "exp_probs_b.bias")
            sel = [f32(sel[e] + bias[e]) for e in range(ne)]
        order = sorted(range(ne), key=lambda e: -sel[e])  # stable sort, descending
        top = order[:k]
        tw = [rw[e] for e in top]
        s = 1e-6
        for w in tw:
            s += w
        inv = 1.0 / s
        rec = [float(e) for e in top] + [f32(w * inv) for w in tw] + rw
        out = [0.0] * c["n_embd"]
        for j, e in enumerate(top):
            if e in self.mask:
                continue
            weight = tw[j] * inv
            g = silu(W.mm(b + "ffn_gate_exps.weight", normed, e))
            g = mul(g, W.mm(b + "ffn_up_exps.weight", normed, e))
            dn = W.mm(b + "ffn_down_exps.weight", g, e)
            out = [f32(out[i] + weight * dn[i]) for i in range(len(out))]
        return out, rec

    def forward(self, token, pos, skip=False):
        W, c = self.W, self.c
        E, eps = c["n_embd"], c["eps"]
        if W.t["token_embd.weight"][0] in KQ_BYTES:  # embeddingLookupGeneric (tensor.js:499-523)
            hidden = column_kq(W.t["token_embd.weight"][0], W.raw("token_embd.weight"), E, token)
        else:
            hidden = embedding_q80(W.raw("token_embd.weight"), E, token)
        recs, hid = [], []
        slot = 0
        for l in range(c["n_layers"]):
            b = f"blk.{l}."
            normed = rmsnorm(hidden, W.f32v(b + "attn_norm.weight"), eps)
            if W.has(b + "shortconv.conv.weight"):
                op = self.shortconv(l, normed)
            else:
                op = self.attention(l, normed, pos, slot)
                slot += 1
            hidden = add(hidden, op)
            normed = rmsnorm(hidden, W.f32v(b + "ffn_norm.weight"), eps)
            if W.has(b + "ffn_gate_inp.weight"):
                out, rec = self.moe(l, normed)
                recs.append(rec)
                hidden = add(hidden, out)
            else:
                g = silu(W.mm(b + "ffn_gate.weight", normed))
                g = mul(g, W.mm(b + "ffn_up.weight", normed))
                hidden = add(hidden, W.mm(b + "ffn_down.weight", g))
            hid.append(list(hidden))
        logits = None
        if not skip:
            h = rmsnorm(hidden, W.f32v(c["out_norm"]), eps)
            out_name = "output.weight" if W.has("output.weight") else "token_embd.weight"
            logits = W.mm(out_name, h)
        return logits, hid, recs


def micro_specs():
    from __graft_entry__ import load_package

    qq3 = load_package()
    S = qq3.synth
    lfm = S.ModelSpec("lfm2moe", 4, 64, 2, 1, 64, 96, 64, 1e6, 1e-5, context_length=128000, attn_layers=(2,),
                      n_expert=8, n_expert_used=4, n_ff_exp=32, n_dense_lead=2, seed=2024, name="micro-lfm2")
    qw = S.ModelSpec("qwen3", 2, 64, 2, 1, 64, 96, 64, 1e6, 1e-6, seed=2025, name="micro-qwen3")
    return qq3, lfm, qw


def micro_qwen3moe_spec(qq3):
    """A micro Qwen3-MoE: every layer attention + an 8-expert, top-2 softmax-routed FFN."""
    return qq3.synth.ModelSpec("qwen3moe", 2, 64, 2, 1, 64, 96, 64, 1e6, 1e-6, n_expert=8, n_expert_used=2,
                               n_ff_exp=32, seed=2026, name="micro-qwen3moe")


def micro_qwen3kq_spec(qq3):
    """A micro Qwen3 (hidden 256) whose embedding / tied lm_head and several projections are k-quants."""
    return qq3.synth.ModelSpec("qwen3", 2, 256, 2, 1, 128, 96, 256, 1e6, 1e-6, seed=2027, name="micro-qwen3-kq")


# tensor -> k-quant type in the micro k-quant model (the rest stay Q8_0 / F32)
KQ_ASSIGN = {"token_embd.weight": 14, "blk.0.attn_q.weight": 12, "blk.0.ffn_down.weight": 14,
             "blk.1.attn_output.weight": 13, "blk.1.ffn_gate.weight": 10, "blk.1.ffn_up.weight": 11}


def kquantize(tensors, seed):
    """Replace the KQ_ASSIGN tensors by seeded random superblocks of their k-quant type (finite,
    small f16 scale fields)."""
    rng = np.random.default_rng(seed)
    d_off = {10: (80, 82), 11: (108,), 12: (0, 2), 13: (0, 2), 14: (208,)}
    out = dict(tensors)
    for name, t in KQ_ASSIGN.items():
        _, ne, _ = tensors[name]
        nblk = ne[1] * -(-ne[0] // QK_K)
        raw = rng.integers(0, 256, size=nblk * KQ_BYTES[t], dtype=np.uint8)
        for b in range(nblk):
            for off in d_off[t]:
                v = np.float16(abs(rng.normal(0, 4e-4)) + 1e-5)
                raw[b * KQ_BYTES[t] + off: b * KQ_BYTES[t] + off + 2] = np.frombuffer(v.tobytes(), np.uint8)
        out[name] = (t, ne, raw)
    return out


def run_model(qq3, spec, tokens, n_gen, tensors=None):
    tensors = tensors if tensors is not None else qq3.synth.build_tensors(spec)
    W = Weights(tensors)
    cfg = dict(n_embd=spec.n_embd, n_head=spec.n_head, n_head_kv=spec.n_head_kv, head_dim=spec.head_dim,
               eps=float(np.float32(spec.eps)), rope=spec.rope_base, n_layers=spec.n_layers,
               n_expert=spec.n_expert, n_used=spec.n_expert_used, arch=spec.arch,
               out_norm="token_embd_norm.weight" if spec.arch == "lfm2moe" else "output_norm.weight")
    eng = Engine(W, cfg)
    logits, hidden, recs = [], [], []
    for p, t in enumerate(tokens):
        lg, hd, rc = eng.forward(int(t), p)
        logits.append(lg)
        hidden.append(hd)
        recs.append(rc)
    # greedy continuation from the last prompt token's logits (generate(), temperature 0)
    gen, cur, pos = [], argmax_first(logits[-1]), len(tokens)
    for _ in range(n_gen):
        lg, _, _ = eng.forward(cur, pos)
        gen.append(cur)
        cur = argmax_first(lg)
        pos += 1
    out = dict(tokens=np.asarray(tokens, np.int32), logits=np.asarray(logits, np.float32),
               hidden=np.asarray(hidden, np.float32), generated=np.asarray(gen, np.int32))
    if recs and recs[0]:
        out["routing"] = np.asarray(recs, np.float32)
    for name, (t, ne, raw) in tensors.items():
        out["w:" + name] = raw
        out["ne:" + name] = np.asarray(ne + [t], np.int64)
    return out


def ops_vectors(qq3):
    S = qq3.synth
    K, N = 96, 10
    raw = S.q8_0_blocks(K * N, seed=31, mode=1)
    x = S.normal_f32(2 * K, seed=32).reshape(2, K)
    y = [matmul_q80(raw.tobytes(), K, N, [float(v) for v in row]) for row in x]
    emb = embedding_q80(raw.tobytes(), K, 7)
    v = [float(t) for t in S.normal_f32(128, seed=33) * 2.0]
    w = [float(t) for t in S.normal_f32(64, seed=34)]
    return dict(mm_raw=raw, mm_x=x, mm_y=np.asarray(y, np.float32), emb=np.asarray(emb, np.float32),
                vec=np.asarray(v, np.float32), w=np.asarray(w, np.float32),
                rms=np.asarray(per_head_rmsnorm(v, 2, 64, w, float(np.float32(1e-6))), np.float32),
                rope=np.asarray(rope(v, 2, 64, 37, 1e6), np.float32),
                softmax=np.asarray(softmax(v), np.float32), silu=np.asarray(silu(v), np.float32),
                greedy=np.asarray([argmax_first(v)], np.int32))


# ---- k-quants (tensor.js:267-664), transcribed type by type -------------------------------

QK_K = 256
KQ_BYTES = {10: 84, 11: 110, 12: 144, 13: 176, 14: 210}


def q4k_get_scale_min(u8, base, sub):
    """_q4kGetScaleMin (tensor.js:278-289)."""
    if sub < 4:
        return u8[base + sub] & 63, u8[base + sub + 4] & 63
    ss = sub - 4
    s = (u8[base + sub + 4] & 0xF) | ((u8[base + ss] >> 6) << 4)
    m = (u8[base + sub + 4] >> 4) | ((u8[base + sub] >> 6) << 4)
    return s, m


def q3k_get_scale(u8, base, sub):
    """_q3kGetScale (tensor.js:295-302)."""
    lo4 = (u8[base + (sub & 7)] >> ((sub >> 3) << 2)) & 0xF
    hi2 = (u8[base + 8 + (sub & 3)] >> ((sub >> 2) * 2)) & 0x3
    return (lo4 | (hi2 << 4)) - 32


def kq_weight(t, u8, bb, e):
    """The per-element weight of matmulQ{2..6}KxF32 (tensor.js:304-466), a JS number."""
    if t == 10:
        d, dmin = read_f16(u8, bb + 80), read_f16(u8, bb + 82)
        sb = u8[bb + (e >> 4)]
        qb = bb + 16 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)
        q = (u8[qb] >> (((e >> 5) & 3) * 2)) & 0x3
        return d * (sb & 0xF) * q - dmin * ((sb >> 4) & 0xF)
    if t == 11:
        d = read_f16(u8, bb + 108)
        scale = q3k_get_scale(u8, bb + 96, e >> 4)
        hbit = (u8[bb + ((e >> 4) & 1) * 16 + (e & 15)] >> (e >> 5)) & 1
        qb = bb + 32 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)
        low2 = (u8[qb] >> (((e >> 5) & 3) * 2)) & 3
        return d * scale * ((low2 | (hbit << 2)) - 4)
    if t == 12:
        d, dmin = read_f16(u8, bb), read_f16(u8, bb + 2)
        sc, mn = q4k_get_scale_min(u8, bb + 4, (e >> 6) * 2 + ((e >> 5) & 1))
        qs = u8[bb + 16 + (e >> 6) * 32 + (e & 31)]
        q4 = (qs >> 4) & 0xF if (e >> 5) & 1 else qs & 0xF
        return d * sc * q4 - dmin * mn
    if t == 13:
        d, dmin = read_f16(u8, bb), read_f16(u8, bb + 2)
        sc, mn = q4k_get_scale_min(u8, bb + 4, (e >> 6) * 2 + ((e >> 5) & 1))
        qh_bit = (e >> 6) * 2 + ((e >> 5) & 1)
        high = (u8[bb + 16 + (e & 31)] >> qh_bit) & 1
        qs = u8[bb + 48 + (e >> 6) * 32 + (e & 31)]
        low4 = (qs >> 4) & 0xF if (e >> 5) & 1 else qs & 0xF
        return d * sc * (low4 | (high << 4)) - dmin * mn
    if t == 14:
        d = read_f16(u8, bb + 208)
        ql = u8[bb + (e >> 7) * 64 + ((e >> 5) & 1) * 32 + (e & 31)]
        low4 = (ql >> 4) & 0xF if (e >> 6) & 1 else ql & 0xF
        qh = u8[bb + 128 + (e >> 7) * 32 + (e & 31)]
        high2 = (qh >> (((e >> 5) & 3) * 2)) & 0x3
        sbyte = u8[bb + 192 + (e >> 7) * 8 + ((e >> 5) & 3) * 2 + ((e & 31) >> 4)]
        scale = sbyte - 256 if sbyte >= 128 else sbyte
        return d * scale * ((low4 | (high2 << 4)) - 32)
    raise ValueError(t)


def matmul_kq(t, w: bytes, in_dim, out_dim, x):
    """matmulQ{2..6}KxF32 (tensor.js:304-466): dot += input * weight, f32 store."""
    bpc = -(-in_dim // QK_K)
    out = []
    for c in range(out_dim):
        dot = 0.0
        for b in range(bpc):
            bb = (c * bpc + b) * KQ_BYTES[t]
            for e in range(min(QK_K, in_dim - b * QK_K)):
                dot += x[b * QK_K + e] * kq_weight(t, w, bb, e)
        out.append(f32(dot))
    return out


def column_kq(t, w: bytes, out_dim, c):
    """_q{2..6}kColumn (tensor.js:551-664): one column stored into a Float32Array."""
    bpc = -(-out_dim // QK_K)
    out = []
    for b in range(bpc):
        bb = (c * bpc + b) * KQ_BYTES[t]
        for e in range(min(QK_K, out_dim - b * QK_K)):
            out.append(f32(kq_weight(t, w, bb, e)))
    return out


def kquant_vectors():
    """Seeded random superblocks of every k-quant type (random bytes, finite f16 scale fields),
    K = 512 and a ragged K = 300 (the last superblock partly used), 4 columns, 2 input rows."""
    rng = np.random.default_rng(2024)
    d_off = {10: (80, 82), 11: (108,), 12: (0, 2), 13: (0, 2), 14: (208,)}
    out = {}
    for t in (10, 11, 12, 13, 14):
        for K in (512, 300):
            N = 4
            nblk = N * -(-K // QK_K)
            raw = rng.integers(0, 256, size=nblk * KQ_BYTES[t], dtype=np.uint8)
            for b in range(nblk):
                for off in d_off[t]:
                    v = np.float16(abs(rng.normal(0, 0.02)) + 1e-4)
                    raw[b * KQ_BYTES[t] + off: b * KQ_BYTES[t] + off + 2] = np.frombuffer(v.tobytes(), np.uint8)
            x = rng.standard_normal((2, K)).astype(np.float32)
            w = raw.tobytes()
            y = [matmul_kq(t, w, K, N, [float(v) for v in row]) for row in x]
            cols = [column_kq(t, w, K, c) for c in range(N)]
            key = f"t{t}_k{K}"
            out[key + "_raw"] = raw
            out[key + "_x"] = x
            out[key + "_y"] = np.asarray(y, np.float32)
            out[key + "_cols"] = np.asarray(cols, np.float32)
    return out


def main():
    qq3, lfm, qw = micro_specs()
    np.savez_compressed(HERE / "ops.npz", **ops_vectors(qq3))
    toks_l = qq3.synth.uniform_tokens(5, 77, lfm.n_vocab)
    np.savez_compressed(HERE / "micro_lfm2.npz", **run_model(qq3, lfm, toks_l, 4))
    toks_q = qq3.synth.uniform_tokens(5, 78, qw.n_vocab)
    np.savez_compressed(HERE / "micro_qwen3.npz", **run_model(qq3, qw, toks_q, 4))
    np.savez_compressed(HERE / "kquants.npz", **kquant_vectors())
    write_qwen3moe(qq3)
    write_qwen3kq(qq3)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


def write_qwen3kq(qq3):
    spec = micro_qwen3kq_spec(qq3)
    toks = qq3.synth.uniform_tokens(4, 80, spec.n_vocab)
    tensors = kquantize(qq3.synth.build_tensors(spec), 2028)
    np.savez_compressed(HERE / "micro_qwen3kq.npz", **run_model(qq3, spec, toks, 3, tensors))


def write_qwen3moe(qq3):
    spec = micro_qwen3moe_spec(qq3)
    toks = qq3.synth.uniform_tokens(5, 79, spec.n_vocab)
    np.savez_compressed(HERE / "micro_qwen3moe.npz", **run_model(qq3, spec, toks, 4))


if __name__ == "__main__":
    # with an argument, only that file (leaves the others as they are)
    if sys.argv[1:] == ["kquants"]:
        np.savez_compressed(HERE / "kquants.npz", **kquant_vectors())
    elif sys.argv[1:] == ["qwen3moe"]:
        write_qwen3moe(micro_specs()[0])
    elif sys.argv[1:] == ["qwen3kq"]:
        write_qwen3kq(micro_specs()[0])
    else:
        main()
