"""Batched fp32 CPU restatement of the DiT velocity forward with PyTorch.

TEST INFRASTRUCTURE / CPU BASELINE ONLY: bench.py's cpu_baseline leg times it
as the batched CPU throughput line (all rows of a batch through MKL GEMMs at
once, all host threads), beside the reference's own per-token path; tests
check it against oracle.c.  The CUDA engine never uses it.

The arithmetic is the reference's (include/dit_manual.h:88-199,
src/e2e_pipeline_v4.cpp:441-478), with the FFN applied to every token as the
model intends, and the half-split RoPE of manual_attention with its angle
recipe (theta advanced by repeated float multiplication).  Weights are the
checkpoint-named float32 arrays of dots.tts.cpp_b200/synth.py."""
from __future__ import annotations

import numpy as np
import torch


def _rope_tables(pos):
    """cos/sin [L][32] of manual_attention's half-split RoPE (dit_manual.h:111-128)."""
    ts = np.float32(np.power(np.float32(10000.0), np.float32(-2.0 / 64.0)))
    theta = np.empty(32, np.float32)
    t = np.float32(1.0)
    for d in range(32):
        theta[d] = t
        t = np.float32(t * ts)
    ang = np.asarray(pos, np.float32)[:, None] * theta[None, :]
    return torch.from_numpy(np.cos(ang)), torch.from_numpy(np.sin(ang))


class BatchedDiT:
    def __init__(self, w: dict, n_layers: int):
        T = lambda n: torch.from_numpy(np.ascontiguousarray(w[n], np.float32))  # noqa: E731
        v = "velocity_field_predictor."
        self.in_w, self.in_b = T(v + "input_layer.weight"), T(v + "input_layer.bias")
        self.oada_w = T(v + "output_layer.adaLN_modulation.1.weight")
        self.oada_b = T(v + "output_layer.adaLN_modulation.1.bias")
        self.out_w, self.out_b = T(v + "output_layer.linear.weight"), T(v + "output_layer.linear.bias")
        self.blocks = []
        for i in range(n_layers):
            p = f"{v}blocks.{i}."
            self.blocks.append({
                "wqkv": torch.cat([T(p + f"attn.{n}_proj.weight") for n in ("q", "k", "v")]),
                "wo": T(p + "attn.o_proj.weight"), "bo": T(p + "attn.o_proj.bias"),
                "qn": T(p + "attn.q_norm.weight"), "kn": T(p + "attn.k_norm.weight"),
                "w1": T(p + "ffn.fc1.weight"), "b1": T(p + "ffn.fc1.bias"),
                "w2": T(p + "ffn.fc2.weight"), "b2": T(p + "ffn.fc2.bias"),
                "ada_w": T(p + "adaLN_modulation.1.weight"), "ada_b": T(p + "adaLN_modulation.1.bias"),
            })

    @staticmethod
    def _ln(x):
        mean = x.mean(-1, keepdim=True)
        var = ((x - mean) ** 2).mean(-1, keepdim=True)
        return (x - mean) / torch.sqrt(var + 1e-5)

    @staticmethod
    def _rms(v, g):
        return v / torch.sqrt((v * v).mean(-1, keepdim=True) + 1e-6) * g

    @torch.no_grad()
    def velocity(self, x_in, cond, mask=None, pos=None, n_out=4):
        """x_in [R][L][1024], cond [R][1024] (raw c), mask [L][L] (1 = attend) or
        None, pos [L] or None -> velocity of the last n_out rows, [R][n_out][128]."""
        x = torch.as_tensor(np.ascontiguousarray(x_in, np.float32))
        c = torch.as_tensor(np.ascontiguousarray(cond, np.float32))
        R, L, D = x.shape
        cs, sn = _rope_tables(np.arange(L, dtype=np.float32) if pos is None else pos)
        keep = None if mask is None else torch.as_tensor(np.asarray(mask, bool))
        sc = torch.nn.functional.silu(c)
        h = x @ self.in_w.T + self.in_b
        for b in self.blocks:
            ada = sc @ b["ada_w"].T + b["ada_b"]
            sm, scm, gm, sml, scl, gml = ada[:, None, :].chunk(6, dim=-1)
            mod = self._ln(h) * (1.0 + scm) + sm
            q, k, v = (mod @ b["wqkv"].T).view(R, L, 3, 16, 64).unbind(2)
            q, k = self._rms(q, b["qn"]), self._rms(k, b["kn"])
            c_, s_ = cs[None, :, None, :], sn[None, :, None, :]
            q = torch.cat([q[..., :32] * c_ - q[..., 32:] * s_, q[..., 32:] * c_ + q[..., :32] * s_], -1)
            k = torch.cat([k[..., :32] * c_ - k[..., 32:] * s_, k[..., 32:] * c_ + k[..., :32] * s_], -1)
            s = torch.einsum("rihd,rjhd->rhij", q, k) / 8.0
            if keep is not None:
                s = s.masked_fill(~keep, float("-inf"))
            ctx = torch.einsum("rhij,rjhd->rihd", torch.softmax(s, -1), v).reshape(R, L, D)
            h = h + gm * (ctx @ b["wo"].T + b["bo"])
            mod = self._ln(h) * (1.0 + scl) + sml
            f = torch.nn.functional.gelu(mod @ b["w1"].T + b["b1"], approximate="tanh")
            h = h + gml * (f @ b["w2"].T + b["b2"])
        shift, scale = (sc @ self.oada_w.T + self.oada_b)[:, None, :].chunk(2, dim=-1)
        y = self._ln(h[:, L - n_out:]) * (1.0 + scale) + shift
        return (y @ self.out_w.T + self.out_b).numpy()
