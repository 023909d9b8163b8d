"""numpy fp32 restatement of the Laya forward pass (test infrastructure; see oracle/__init__.py).

One question = one sequence, processed on its own: in the reference every padded position is
masked as a key (ModernBERT attention mask, and ``src_key_padding_mask`` in the head), so a
question's outputs do not depend on the rest of its batch. Follows, step by step:

  encoder      transformers ModernBertModel (modeling_modernbert.py: embeddings tok_emb -> LayerNorm;
               pre-LN layers with Identity attn_norm at layer 0; fused Wqkv; HF rotate_half RoPE with
               inv_freq = 1/theta^(2i/64) in fp32, theta by layer type; bidirectional attention, sliding
               layers restricted to |q-k| <= local_attention/2; GeGLU MLP input*gelu(erf) gate from
               Wi.chunk(2); final_norm)
  decision     ref/rl_common.py:100-124 DecisionModel.forward: + type_emb[qtype] on every row;
               head = nn.TransformerEncoderLayer(norm_first, ReLU FFN 4d, biased, nhead d/64);
               scorer LN -> Linear -> GELU -> Linear(d,1) at every marker; act head on the CLS row with
               features [top1, top1-top2, entropy/log(max(k,2)), max(k,2)/255] of softmax(logits).

For a question with one marker the reference model would call topk(2) on a 1-wide tensor (only when
every question of its batch has one option); the reference engine defines top2 = 0 there
(src/kernels.hip:290-297) and so does this oracle.
"""
import math
from typing import Dict, List, Optional

import numpy as np

try:
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)

F32 = np.float32


def gelu(x):
    return (F32(0.5) * x * (F32(1.0) + _erf(x * F32(1.0 / math.sqrt(2.0))).astype(F32))).astype(F32)


def layer_norm(x, w, b=None, eps=1e-5):
    mu = x.mean(-1, keepdims=True, dtype=F32)
    xc = x - mu
    var = (xc * xc).mean(-1, keepdims=True, dtype=F32)
    y = xc / np.sqrt(var + F32(eps)) * w
    if b is not None:
        y = y + b
    return y.astype(F32)


def rope_tables(L, theta, hd=64):
    """cos/sin [L, hd] as transformers computes them (fp32 inv_freq, fp32 product, cat(freqs, freqs))."""
    inv = (F32(1.0) / (F32(theta) ** (np.arange(0, hd, 2, dtype=np.int64).astype(F32) / F32(hd)))).astype(F32)
    f = (np.arange(L, dtype=F32)[:, None] * inv[None, :]).astype(F32)
    emb = np.concatenate([f, f], -1)
    return np.cos(emb.astype(np.float64)).astype(F32), np.sin(emb.astype(np.float64)).astype(F32)


def rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], -1)


def attention(q, k, v, window=None):
    """q,k,v [H, L, hd]; bidirectional softmax(q k^T / sqrt(hd)) v, optional |i-j| <= window band."""
    hd = q.shape[-1]
    s = np.matmul(q, k.transpose(0, 2, 1)) * F32(1.0 / math.sqrt(hd))
    if window is not None:
        L = q.shape[1]
        i = np.arange(L)
        s = np.where(np.abs(i[:, None] - i[None, :]) <= window, s, F32(-np.inf))
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return np.matmul(p.astype(F32), v).astype(F32)


class Oracle:
    """Holds one checkpoint's weights (fp32) and runs questions through the reference forward."""

    def __init__(self, weights: Dict[str, np.ndarray], arch):
        self.w = {k: np.ascontiguousarray(v, dtype=F32) for k, v in weights.items()}
        self.a = arch
        self.layer_types = getattr(arch, "_layer_types", None) or arch.layer_types()
        self._rope = {}

    def _tables(self, L, theta):
        key = (L, theta)
        if key not in self._rope:
            self._rope[key] = rope_tables(L, theta)
        return self._rope[key]

    def encoder(self, ids, capture: Optional[dict] = None):
        a, w = self.a, self.w
        D, H = a.d, a.heads
        hd = D // H
        L = len(ids)
        h = layer_norm(w["encoder.embeddings.tok_embeddings.weight"][np.asarray(ids)],
                       w["encoder.embeddings.norm.weight"], eps=a.eps)
        if capture is not None:
            capture["emb"] = h.copy()
        for i in range(a.layers):
            p = "encoder.layers.%d." % i
            x = h if i == 0 else layer_norm(h, w[p + "attn_norm.weight"], eps=a.eps)
            qkv = (x @ w[p + "attn.Wqkv.weight"].T).reshape(L, 3, H, hd).transpose(1, 2, 0, 3)
            q, k, v = qkv[0], qkv[1], qkv[2]
            glob = self.layer_types[i] == "full_attention"
            cos, sin = self._tables(L, a.theta_global if glob else a.theta_local)
            q = (q * cos + rotate_half(q) * sin).astype(F32)
            k = (k * cos + rotate_half(k) * sin).astype(F32)
            o = attention(q, k, v, None if glob else a.local_attention // 2)
            h = (h + o.transpose(1, 0, 2).reshape(L, D) @ w[p + "attn.Wo.weight"].T).astype(F32)
            m = layer_norm(h, w[p + "mlp_norm.weight"], eps=a.eps)
            u = m @ w[p + "mlp.Wi.weight"].T
            g = gelu(u[:, :a.inter]) * u[:, a.inter:]
            h = (h + g @ w[p + "mlp.Wo.weight"].T).astype(F32)
            if capture is not None:
                capture["enc%d" % i] = h.copy()
        h = layer_norm(h, w["encoder.final_norm.weight"], eps=a.eps)
        if capture is not None:
            capture["final_norm"] = h.copy()
        return h

    def head_layer(self, j, h):
        a, w = self.a, self.w
        D = a.d
        H = max(1, D // 64)
        hd = D // H
        L = h.shape[0]
        p = "head.layers.%d." % j
        x = layer_norm(h, w[p + "norm1.weight"], w[p + "norm1.bias"], eps=1e-5)
        qkv = (x @ w[p + "self_attn.in_proj_weight"].T + w[p + "self_attn.in_proj_bias"]).astype(F32)
        qkv = qkv.reshape(L, 3, H, hd).transpose(1, 2, 0, 3)
        o = attention(qkv[0], qkv[1], qkv[2], None).transpose(1, 0, 2).reshape(L, D)
        h = (h + o @ w[p + "self_attn.out_proj.weight"].T + w[p + "self_attn.out_proj.bias"]).astype(F32)
        x = layer_norm(h, w[p + "norm2.weight"], w[p + "norm2.bias"], eps=1e-5)
        f = np.maximum(x @ w[p + "linear1.weight"].T + w[p + "linear1.bias"], F32(0))
        return (h + f @ w[p + "linear2.weight"].T + w[p + "linear2.bias"]).astype(F32)

    def forward_one(self, ids, markers, qtype, capture: Optional[dict] = None):
        """Returns (logits[k], act_logits[n_act]) of one question; fills `capture` with per-layer rows."""
        a, w = self.a, self.w
        h = self.encoder(ids, capture)
        h = (h + w["type_emb.weight"][qtype]).astype(F32)
        if capture is not None:
            capture["final"] = h.copy()
        for j in range(a.head_layers):
            h = self.head_layer(j, h)
            if capture is not None:
                capture["head%d" % j] = h.copy()
        m = h[np.asarray(markers)]
        z = layer_norm(m, w["scorer.0.weight"], w["scorer.0.bias"], eps=1e-5)
        z = gelu((z @ w["scorer.1.weight"].T + w["scorer.1.bias"]).astype(F32))
        logits = (z @ w["scorer.3.weight"].T + w["scorer.3.bias"]).astype(F32)[:, 0]
        act = self.act_head(h[0], logits)
        return logits, act

    def act_head(self, cls_row, logits):
        w = self.w
        z = logits.astype(F32)
        e = np.exp(z - z.max())
        p = (e / e.sum()).astype(F32)
        K = len(z)
        k = F32(max(K, 2))
        ent = -(p * np.log(np.maximum(p, F32(1e-9)))).sum(dtype=F32) / np.log(k)
        srt = np.sort(p)[::-1]
        t1 = srt[0]
        t2 = srt[1] if K > 1 else F32(0)
        feats = np.array([t1, t1 - t2, ent, k / F32(255.0)], dtype=F32)
        x = np.concatenate([cls_row.astype(F32), feats])
        hid = gelu((w["act_head.0.weight"] @ x + w["act_head.0.bias"]).astype(F32))
        return (w["act_head.2.weight"] @ hid + w["act_head.2.bias"]).astype(F32)

    def forward_batch(self, questions: List[dict], capture: bool = False):
        """questions: dicts with ids, markers, qtype. Returns (logits concatenated, act [B, n_act], caps)."""
        los, acts, caps = [], [], []
        for q in questions:
            c = {} if capture else None
            lo, ac = self.forward_one(q["ids"], q["markers"], q["qtype"], c)
            los.append(lo)
            acts.append(ac)
            caps.append(c)
        return np.concatenate(los) if los else np.zeros(0, F32), np.stack(acts), caps


def softmax(z, T=1.0):
    z = np.asarray(z, dtype=np.float64) / T
    e = np.exp(z - z.max())
    return e / e.sum()
