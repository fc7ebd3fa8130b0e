"""Qwen2.5-1.5B decoder prefill and KV-cache step: numpy fp32 restatement of the
reference's own LLM path.

TEST INFRASTRUCTURE ONLY: tests/ use it as a checker (it is pinned against the
reference build in oracle/_ref and against tests/golden/llm_ref_small.npz);
the CUDA engine never routes through it.

The reference follows, step by step:
  llm_manual_forward   src/llm_manual.cpp:61-176   prefill hidden states
  llm_kv_cache_init    src/llm_manual.cpp:237-340  K (rotated) and V cached per layer
  llm_kv_cache_step    src/llm_manual.cpp:342-475  one token against the cache
  manual_rms_norm      include/dit_manual.h:23-27  x / sqrt(sum(x^2)/n + 1e-6) * w
  manual_linear        include/dit_manual.h:30-61  W x + b in fp32 loops (LLM sizes)
  manual_rope_theta    include/dit_manual.h:63-78  half-split pairs (d, d + 64),
                       theta advanced by repeated float multiplication, base 1e6
  manual_softmax       include/dit_manual.h:83-86  max-subtracted expf, divided by the sum
Grouped-query attention maps query head h to KV head h * 2 / 12
(src/llm_manual.cpp:117, 362).  The gate of the MLP is SiLU written as
g / (1 + e^-g) (:163, :454).  The final norm uses llm.model.norm.weight.

Weights are the checkpoint-named float32 arrays of dots.tts.cpp_b200/synth.py
(src/llm_manual.cpp:26-44).  The reference's summation order is sequential;
numpy's is pairwise, so agreement is to fp32 rounding, not bitwise."""
from __future__ import annotations

import numpy as np

H, F, NH, NKV, HD = 1536, 8960, 12, 2, 128
ROPE_BASE = 1000000.0
EPS = 1e-6

_f = np.float32


def rms_norm(x, g):
    """include/dit_manual.h:23-27, row by row."""
    x = np.asarray(x, _f)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=_f)
    inv = _f(1.0) / np.sqrt(ss / _f(x.shape[-1]) + _f(EPS))
    return (x * inv) * np.asarray(g, _f)


def rope_tables(pos):
    """cos, sin [len(pos)][64] of manual_rope_theta (include/dit_manual.h:63-78):
    theta_0 = 1, theta_{d+1} = theta_d * 1e6^(-2/128) in float; angle = pos * theta_d."""
    ts = _f(np.power(_f(ROPE_BASE), _f(-2.0 / HD)))
    theta = np.empty(HD // 2, _f)
    t = _f(1.0)
    for d in range(HD // 2):
        theta[d] = t
        t = _f(t * ts)
    ang = np.asarray(pos, _f)[:, None] * theta[None, :]
    return np.cos(ang).astype(_f), np.sin(ang).astype(_f)


def rope(x, cs, sn):
    """Rotate [T][heads][128] at the positions of (cs, sn) [T][64]: pairs (d, d + 64)."""
    c, s = cs[:, None, :], sn[:, None, :]
    a, b = x[..., :HD // 2], x[..., HD // 2:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


def softmax_rows(s):
    """include/dit_manual.h:83-86 on every row (-inf entries give 0)."""
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m).astype(_f)
    return e / np.sum(e, axis=-1, keepdims=True, dtype=_f)


class LLMOracle:
    """Prefill then steps on one sequence, keeping the reference's cache layout in
    spirit: per layer, K rotated at its own position and V as projected."""

    def __init__(self, w: dict, n_layers: int):
        A = lambda n: np.ascontiguousarray(w[n], _f)  # noqa: E731
        self.layers = []
        for i in range(n_layers):
            p = f"llm.model.layers.{i}."
            self.layers.append({
                "an": A(p + "input_layernorm.weight"), "fn": A(p + "post_attention_layernorm.weight"),
                "qw": A(p + "self_attn.q_proj.weight"), "qb": A(p + "self_attn.q_proj.bias"),
                "kw": A(p + "self_attn.k_proj.weight"), "kb": A(p + "self_attn.k_proj.bias"),
                "vw": A(p + "self_attn.v_proj.weight"), "vb": A(p + "self_attn.v_proj.bias"),
                "ow": A(p + "self_attn.o_proj.weight"),
                "gw": A(p + "mlp.gate_proj.weight"), "uw": A(p + "mlp.up_proj.weight"),
                "dw": A(p + "mlp.down_proj.weight"),
            })
        self.final = A("llm.model.norm.weight")
        self.k = [None] * n_layers   # [T][2][128], rotated
        self.v = [None] * n_layers   # [T][2][128]
        self.length = 0

    def _layers(self, h, pos):
        """Run every layer on new tokens h [T][1536] at positions pos, attending to
        the cache plus themselves causally; appends to the cache."""
        T = h.shape[0]
        cs, sn = rope_tables(pos)
        for i, l in enumerate(self.layers):
            x = rms_norm(h, l["an"])
            q = (x @ l["qw"].T + l["qb"]).reshape(T, NH, HD)
            k = (x @ l["kw"].T + l["kb"]).reshape(T, NKV, HD)
            v = (x @ l["vw"].T + l["vb"]).reshape(T, NKV, HD)
            q, k = rope(q, cs, sn), rope(k, cs, sn)
            kc = k if self.k[i] is None else np.concatenate([self.k[i], k])
            vc = v if self.v[i] is None else np.concatenate([self.v[i], v])
            self.k[i], self.v[i] = kc, vc
            S = kc.shape[0]
            ao = np.empty((T, NH, HD), _f)
            causal = np.arange(S)[None, :] > (S - T + np.arange(T))[:, None]
            for hq in range(NH):
                kv = hq * NKV // NH
                s = (q[:, hq, :] @ kc[:, kv, :].T) * _f(1.0 / np.sqrt(_f(HD)))
                s = np.where(causal, _f(-np.inf), s).astype(_f)
                ao[:, hq, :] = softmax_rows(s) @ vc[:, kv, :]
            h2 = h + ao.reshape(T, H) @ l["ow"].T
            x = rms_norm(h2, l["fn"])
            g = x @ l["gw"].T
            u = x @ l["uw"].T
            a = (g / (_f(1.0) + np.exp(-g))) * u
            h = h2 + a @ l["dw"].T
        self.length += T
        return rms_norm(h, self.final)

    def prefill(self, emb):
        """emb [n_tok][1536] -> final-normed hidden [n_tok][1536] (llm_kv_cache_init)."""
        emb = np.asarray(emb, _f)
        assert self.length == 0, "prefill starts an empty cache"
        return self._layers(emb, np.arange(emb.shape[0]))

    def step(self, emb_row):
        """One embedding [1536] at position = cache length -> hidden [1536] (llm_kv_cache_step)."""
        x = np.asarray(emb_row, _f)[None, :]
        return self._layers(x, np.array([self.length]))[0]


def run(w, n_layers, prompt_emb, step_emb):
    """Same contract as the reference driver's ref_llm_run: the prompt's hidden
    states [n_tok][1536] and one hidden state per row of step_emb."""
    o = LLMOracle(w, n_layers)
    ph = o.prefill(prompt_emb)
    sh = np.stack([o.step(e) for e in np.asarray(step_emb, _f)]) if len(step_emb) else np.zeros((0, H), _f)
    return ph, sh
