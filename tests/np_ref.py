"""Independent float64 numpy restatement of the talker step and the predictor
frame (talker.rs:263-360, code_predictor.rs:218-513).

Second, independent implementation used only to cross-check the C oracle's
indexing at model level (the reference has no model-level golden vectors).
Written from the reference's algorithm, not from the oracle's C code.
"""
import numpy as np


def deq(w):
    """Dequantise a Q4Weight to float64 [k][n] (gemv.rs:18-31 layout)."""
    k, n = w.k, w.n
    p = w.packed.reshape(k, n // 32, 16)
    lo = (p & 15).astype(np.int64) - 8
    hi = (p >> 4).astype(np.int64) - 8
    q = np.stack([lo, hi], -1).reshape(k, n)
    sc = w.scales.view(np.float16).astype(np.float64).reshape(k, n // 32)
    return q * np.repeat(sc, 32, axis=1)


def f16(a):
    return a.view(np.float16).astype(np.float64)


def rms(x, g):
    return x / np.sqrt(np.mean(x * x) + 1e-6) * f16(g)


def qknorm(v, heads, hd, g):
    v = v.reshape(heads, hd)
    return (v / np.sqrt(np.mean(v * v, axis=1, keepdims=True) + 1e-6) * f16(g)).reshape(-1)


def rope(v, heads, hd, pos, theta=1e6):
    half = hd // 2
    i = np.arange(half)
    freq = 1.0 / theta ** (2 * i / hd)
    c, s = np.cos(pos * freq), np.sin(pos * freq)
    v = v.reshape(heads, hd).copy()
    x1, x2 = v[:, :half].copy(), v[:, half:].copy()
    v[:, :half] = x1 * c - x2 * s
    v[:, half:] = x2 * c + x1 * s
    return v.reshape(-1)


def silu(x):
    return x / (1 + np.exp(-x))


def embed_text_token(tp, token):
    """embed_text_token (talker.rs:104-116) in float64: text-embedding row ->
    fc1 + bias -> SiLU -> fc2 + bias."""
    raw = deq(tp.text_embedding)[token] if tp.text_embedding.k < 4096 else None
    if raw is None:  # large tables: dequantise the one row
        e = tp.text_embedding
        g = e.n // 32
        p = e.packed.reshape(e.k, g, 16)[token]
        q = np.stack([(p & 15).astype(np.int64) - 8, (p >> 4).astype(np.int64) - 8], -1).reshape(-1)
        raw = q * np.repeat(e.scales.view(np.float16).astype(np.float64).reshape(e.k, g)[token], 32)
    h = silu(raw @ deq(tp.fc1) + tp.fc1_bias.astype(np.float64))
    return h @ deq(tp.fc2) + tp.fc2_bias.astype(np.float64)


class NpKV:
    def __init__(self, layers):
        self.k = [[] for _ in range(layers)]
        self.v = [[] for _ in range(layers)]


def layer_step(lw, W, x, kvk, kvv, pos, heads, kvh, hd):
    xn = rms(x, lw.input_norm)
    q = xn @ W["q"]
    k = xn @ W["k"]
    v = xn @ W["v"]
    q = rope(qknorm(q, heads, hd, lw.q_norm), heads, hd, pos)
    k = rope(qknorm(k, kvh, hd, lw.k_norm), kvh, hd, pos)
    kvk.append(k.reshape(kvh, hd))
    kvv.append(v.reshape(kvh, hd))
    K = np.stack(kvk)
    V = np.stack(kvv)
    out = np.zeros(heads * hd)
    g = heads // kvh
    for h in range(heads):
        sc = K[:, h // g] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        p /= p.sum()
        out[h * hd:(h + 1) * hd] = p @ V[:, h // g]
    x = x + out @ W["o"]
    xn = rms(x, lw.post_attn_norm)
    x = x + (silu(xn @ W["gate"]) * (xn @ W["up"])) @ W["down"]
    return x


def deq_layer(lw):
    return {"q": deq(lw.q_proj), "k": deq(lw.k_proj), "v": deq(lw.v_proj), "o": deq(lw.o_proj),
            "gate": deq(lw.gate_proj), "up": deq(lw.up_proj), "down": deq(lw.down_proj)}


class NpModel:
    def __init__(self, m):
        self.m = m
        c = m.cfg
        self.tW = [deq_layer(lw) for lw in m.t_layers]
        self.pW = [deq_layer(lw) for lw in m.p_layers]
        self.head = deq(m.codec_head)
        self.cemb = deq(m.codec_embedding)
        self.proj = deq(m.input_proj) if m.input_proj is not None else None
        self.bias = m.input_proj_bias.astype(np.float64) if m.input_proj_bias is not None else None
        self.pemb = [deq(e) for e in m.codec_embeddings]
        self.heads = [deq(h) for h in m.lm_heads]
        self.c = c

    def talker_step(self, emb, kv, pos):
        c = self.c
        x = emb.astype(np.float64)
        for i, lw in enumerate(self.m.t_layers):
            x = layer_step(lw, self.tW[i], x, kv.k[i], kv.v[i], pos, c.t_heads, c.t_kv_heads,
                           c.t_head_dim)
        h = rms(x, self.m.t_final_norm)
        return h, h @ self.head

    def project(self, v):
        if self.proj is None:
            return v
        return v @ self.proj + self.bias

    def predictor_frame(self, hidden, sem, forced=None):
        c = self.c
        kv = NpKV(c.p_layers)
        codes, logits = [], []
        xs = [self.project(hidden.astype(np.float64)), self.project(sem.astype(np.float64))]
        for t, x in enumerate(xs):  # 2-token prefill == two causal decode steps
            for i, lw in enumerate(self.m.p_layers):
                x = layer_step(lw, self.pW[i], x, kv.k[i], kv.v[i], t, c.p_heads, c.p_kv_heads,
                               c.p_head_dim)
        lg = rms(x, self.m.p_final_norm) @ self.heads[0]
        logits.append(lg)
        codes.append(int(np.argmax(lg)))
        for g in range(1, c.p_groups):
            prev = forced[g - 1] if forced is not None else codes[-1]
            x = self.project(self.pemb[g - 1][prev])
            for i, lw in enumerate(self.m.p_layers):
                x = layer_step(lw, self.pW[i], x, kv.k[i], kv.v[i], g + 1, c.p_heads, c.p_kv_heads,
                               c.p_head_dim)
            lg = rms(x, self.m.p_final_norm) @ self.heads[g]
            logits.append(lg)
            codes.append(int(np.argmax(lg)))
        return np.array(codes), np.stack(logits)
