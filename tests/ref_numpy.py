"""Float64 NumPy restatement of the reference decode math (src/gemv.rs:744-1019) used to
cross-check the C++ oracle on small models. Independent of the oracle's code: dense
dequantised weights, plain matrix products, float64 throughout."""
from __future__ import annotations

import numpy as np


class RefModel:
    def __init__(self, model, qf, kv_f16=False):
        """kv_f16: the opt-in binary16 cache: K and V rounded to float16 as they enter it."""
        self.m = model
        self.qf = qf
        self.kv_f16 = kv_f16
        deq = (lambda mat: qf.dequant_q4(mat, np.float64)) if model.format == qf.FORMAT_Q4 else \
            (lambda mat: qf.f16_bits_to_f32(mat.data).astype(np.float64).reshape(mat.k, mat.n))
        self.layers = []
        for L in model.layers:
            self.layers.append(dict(
                W=[deq(m) for m in L.mats()],
                g1=qf.f16_bits_to_f32(L.input_norm_gamma).astype(np.float64),
                g2=qf.f16_bits_to_f32(L.post_attn_norm_gamma).astype(np.float64),
                nh=L.num_heads, nkv=L.num_kv_heads, hd=L.head_dim, grp=L.num_kv_groups))
        self.E = deq(model.embed)
        self.gf = qf.f16_bits_to_f32(model.final_norm_gamma).astype(np.float64)
        half = model.rope_half_dim
        self.cos = model.rope_cos.astype(np.float64).reshape(-1, half)
        self.sin = model.rope_sin.astype(np.float64).reshape(-1, half)

    @staticmethod
    def rms(x, g):
        return x / np.sqrt(np.mean(x * x) + 1e-6) * g

    def rope(self, v, heads, hd, pos):
        v = v.reshape(heads, hd).copy()
        h = hd // 2
        c, s = self.cos[pos], self.sin[pos]
        a, b = v[:, :h].copy(), v[:, h:].copy()
        v[:, :h] = a * c - b * s
        v[:, h:] = b * c + a * s
        return v.reshape(-1)

    def new_kv(self):
        return [([], []) for _ in self.layers]

    def layer(self, i, x, kv):
        L = self.layers[i]
        Wq, Wk, Wv, Wo, Wg, Wu, Wd = L["W"]
        xn = self.rms(x, L["g1"])
        q, k, v = xn @ Wq, xn @ Wk, xn @ Wv
        pos = len(kv[i][0])
        if self.m.no_rope_layers[i]:
            q = self.rope(q, L["nh"], L["hd"], pos)
            k = self.rope(k, L["nkv"], L["hd"], pos)
        if self.kv_f16:
            k = k.astype(np.float16).astype(np.float64)
            v = v.astype(np.float16).astype(np.float64)
        kv[i][0].append(k)
        kv[i][1].append(v)
        K = np.stack(kv[i][0]).reshape(pos + 1, L["nkv"], L["hd"])
        V = np.stack(kv[i][1]).reshape(pos + 1, L["nkv"], L["hd"])
        out = np.zeros((L["nh"], L["hd"]))
        qh = q.reshape(L["nh"], L["hd"])
        for h in range(L["nh"]):
            j = h // L["grp"]
            s = K[:, j, :] @ qh[h] / np.sqrt(L["hd"])
            p = np.exp(s - s.max())
            p /= p.sum()
            out[h] = p @ V[:, j, :]
        x = x + out.reshape(-1) @ Wo
        xn = self.rms(x, L["g2"])
        g, u = xn @ Wg, xn @ Wu
        x = x + (g / (1 + np.exp(-g)) * u) @ Wd
        return x

    def decode(self, token, kv):
        x = self.E[token].copy()
        for i in range(len(self.layers)):
            x = self.layer(i, x, kv)
        return self.E @ self.rms(x, self.gf)
