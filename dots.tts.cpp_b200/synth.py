"""Seeded synthetic weights and inputs in the reference's checkpoint layout.

No checkpoint of the real model is available, so every workload runs on
random-init weights of the real architecture: matrices and biases drawn from
N(0, 0.02), norm gains from 1 + N(0, 0.02).  Tensor names and shapes are the
reference's safetensors names (src/utils/dit_loader.cpp:47-115,
src/utils/patchenc_loader.cpp:175-208); shapes are PyTorch [out, in].

Each tensor gets its own generator seeded by (seed, crc32(name)), so a
2-layer test model is exactly the first two layers of the 18-layer one."""
from __future__ import annotations

import zlib

import numpy as np

D, H, HD, F, LAT, LLM, SPK = 1024, 16, 64, 4096, 128, 1536, 512
DIT_LAYERS, PE_LAYERS = 18, 24


def _rng(seed: int, name: str):
    return np.random.default_rng([int(seed), zlib.crc32(name.encode())])


def normal(seed, name, shape, std=0.02, mean=0.0):
    a = _rng(seed, name).standard_normal(size=shape, dtype=np.float32)
    if std != 1.0:
        a *= np.float32(std)
    if mean != 0.0:
        a += np.float32(mean)
    return a


def dit_shapes(n_layers=DIT_LAYERS):
    s = {}
    for i in range(n_layers):
        p = f"velocity_field_predictor.blocks.{i}."
        for n in ("q", "k", "v", "o"):
            s[p + f"attn.{n}_proj.weight"] = (D, D)
        s[p + "attn.o_proj.bias"] = (D,)
        s[p + "attn.q_norm.weight"] = (HD,)
        s[p + "attn.k_norm.weight"] = (HD,)
        s[p + "ffn.fc1.weight"] = (F, D)
        s[p + "ffn.fc1.bias"] = (F,)
        s[p + "ffn.fc2.weight"] = (D, F)
        s[p + "ffn.fc2.bias"] = (D,)
        s[p + "adaLN_modulation.1.weight"] = (6 * D, D)
        s[p + "adaLN_modulation.1.bias"] = (6 * D,)
    v = "velocity_field_predictor."
    s[v + "time_embedder.mlp.0.weight"] = (D, 256)
    s[v + "time_embedder.mlp.0.bias"] = (D,)
    s[v + "time_embedder.mlp.2.weight"] = (D, D)
    s[v + "time_embedder.mlp.2.bias"] = (D,)
    s["xvec_proj.0.weight"] = (D, SPK)
    s["xvec_proj.0.bias"] = (D,)
    s["xvec_proj.1.weight"] = (D,)
    s["xvec_proj.1.bias"] = (D,)
    s[v + "output_layer.adaLN_modulation.1.weight"] = (2 * D, D)
    s[v + "output_layer.adaLN_modulation.1.bias"] = (2 * D,)
    s[v + "output_layer.linear.weight"] = (LAT, D)
    s[v + "output_layer.linear.bias"] = (LAT,)
    s[v + "input_layer.weight"] = (D, D)
    s[v + "input_layer.bias"] = (D,)
    s["hidden_proj.weight"] = (D, LLM)
    s["hidden_proj.bias"] = (D,)
    s["latent_proj.weight"] = (D, LAT)
    s["latent_proj.bias"] = (D,)
    s["coordinate_proj.weight"] = (D, LAT)
    s["coordinate_proj.bias"] = (D,)
    s["eos_proj.0.weight"] = (LLM, LLM)
    s["eos_proj.0.bias"] = (LLM,)
    s["eos_proj.2.weight"] = (2, LLM)
    s["eos_proj.2.bias"] = (2,)
    return s


def pe_shapes(n_layers=PE_LAYERS):
    s = {}
    for i in range(n_layers):
        p = f"patch_encoder.encoder.layers.{i}."
        for n in ("q", "k", "v", "o"):
            s[p + f"attn.{n}_proj.weight"] = (D, D)
        s[p + "attn.o_proj.bias"] = (D,)
        s[p + "attn_norm.weight"] = (D,)
        s[p + "ffn_norm.weight"] = (D,)
        s[p + "ffn.fc1.weight"] = (F, D)
        s[p + "ffn.fc1.bias"] = (F,)
        s[p + "ffn.fc2.weight"] = (D, F)
        s[p + "ffn.fc2.bias"] = (D,)
    s["patch_encoder.ds_proj.weight"] = (LAT, LAT, 2)
    s["patch_encoder.ds_proj.bias"] = (LAT,)
    s["patch_encoder.in_proj.weight"] = (D, LAT)
    s["patch_encoder.in_proj.bias"] = (D,)
    s["patch_encoder.out_proj.weight"] = (LLM, 2 * D)
    s["patch_encoder.out_proj.bias"] = (LLM,)
    return s


def _is_gain(name):
    return name.endswith(("q_norm.weight", "k_norm.weight", "xvec_proj.1.weight",
                          "attn_norm.weight", "ffn_norm.weight"))


def dit_weights(seed=1, n_layers=DIT_LAYERS, ada_bias_std=0.02):
    """DiT weights.  ada_bias_std > 0.02 makes shift/scale/gate O(1) so that the
    attention and FFN branches dominate a block's output (used by block tests)."""
    w = {}
    for name, shape in dit_shapes(n_layers).items():
        if _is_gain(name):
            w[name] = normal(seed, name, shape, 0.02, 1.0)
        elif name.endswith("adaLN_modulation.1.bias"):
            w[name] = normal(seed, name, shape, ada_bias_std)
        else:
            w[name] = normal(seed, name, shape, 0.02)
    return w


def pe_weights(seed=2, n_layers=PE_LAYERS):
    w = {}
    for name, shape in pe_shapes(n_layers).items():
        w[name] = normal(seed, name, shape, 0.02, 1.0 if _is_gain(name) else 0.0)
    return w


def fm_history(seed, n_utt, fm_len, w=None, hidden_every=5):
    """FM history buffers like src/e2e_pipeline_v4.cpp:331-340,551-588: a
    hidden_proj row at every position p with p % hidden_every == 0 (from
    h ~ N(0,1) [1536]; the unconditional buffer uses hidden_proj(0)) and
    latent_proj rows of z ~ N(0,1) [128] elsewhere (shared by both buffers).
    Projections are computed in fp64 and rounded to fp32 (inputs, not the
    path under test).  Returns (fm_cond, fm_uncond), each [n_utt][fm_len][1024]."""
    hw, hb = w["hidden_proj.weight"].astype(np.float64), w["hidden_proj.bias"].astype(np.float64)
    lw, lb = w["latent_proj.weight"].astype(np.float64), w["latent_proj.bias"].astype(np.float64)
    hid = normal(seed, "fm.hidden", (n_utt, fm_len, LLM), 1.0).astype(np.float64)
    lat = normal(seed, "fm.latent", (n_utt, fm_len, LAT), 1.0).astype(np.float64)
    is_hidden = (np.arange(fm_len) % hidden_every) == 0
    hproj = hid @ hw.T + hb
    lproj = lat @ lw.T + lb
    cond = np.where(is_hidden[None, :, None], hproj, lproj).astype(np.float32)
    null_h = np.broadcast_to(hb, (n_utt, fm_len, D))
    uncond = np.where(is_hidden[None, :, None], null_h, lproj).astype(np.float32)
    return np.ascontiguousarray(cond), np.ascontiguousarray(uncond)


LH, LF, LKV = 1536, 8960, 256          # Qwen2.5-1.5B: hidden, MLP, K/V width (2 heads x 128)
LLM_LAYERS = 28


def llm_shapes(n_layers=LLM_LAYERS):
    """Tensor names and shapes of the LLM's decoder (src/llm_manual.cpp:26-44)."""
    s = {}
    for i in range(n_layers):
        p = f"llm.model.layers.{i}."
        s[p + "input_layernorm.weight"] = (LH,)
        s[p + "post_attention_layernorm.weight"] = (LH,)
        s[p + "self_attn.q_proj.weight"] = (LH, LH)
        s[p + "self_attn.q_proj.bias"] = (LH,)
        s[p + "self_attn.k_proj.weight"] = (LKV, LH)
        s[p + "self_attn.k_proj.bias"] = (LKV,)
        s[p + "self_attn.v_proj.weight"] = (LKV, LH)
        s[p + "self_attn.v_proj.bias"] = (LKV,)
        s[p + "self_attn.o_proj.weight"] = (LH, LH)
        s[p + "mlp.gate_proj.weight"] = (LF, LH)
        s[p + "mlp.up_proj.weight"] = (LF, LH)
        s[p + "mlp.down_proj.weight"] = (LH, LF)
    s["llm.model.norm.weight"] = (LH,)
    return s


def llm_weights(seed=3, n_layers=LLM_LAYERS):
    """LLM decoder weights: N(0, 0.02), norm gains 1 + N(0, 0.02)."""
    w = {}
    for name, shape in llm_shapes(n_layers).items():
        gain = name.endswith("norm.weight")
        w[name] = normal(seed, name, shape, 0.02, 1.0 if gain else 0.0)
    return w


# ---------------------------------------------------------------- vocoder
VOC_UP_IN = (1536, 768, 384, 192, 96, 48)
VOC_UP_OUT = (768, 384, 192, 96, 48, 24)
VOC_UP_STRIDE = (10, 6, 4, 2, 2, 2)
VOC_UP_KERNEL = (20, 12, 8, 4, 4, 4)
VOC_RB_KERNEL = (3, 7, 11)
VOC_RB_DIL = (1, 3, 5)
VOC_HOP = 1920


def voc_shapes():
    """Tensor names and shapes of the BigVGAN decoder checkpoint
    (src/modules/vocoder/bigvgan_cpp.cpp:203-290)."""
    s = {"post_proj.weight": (LAT, LAT, 1), "post_proj.bias": (LAT,),
         "dec_mi_layer.0.weight": (512, LAT), "dec_mi_layer.0.bias": (512,),
         "dec_mi_layer.2.weight": (LAT, 512), "dec_mi_layer.2.bias": (LAT,),
         "decoder.conv_pre.weight": (1536, LAT, 5), "decoder.conv_pre.bias": (1536,)}
    for l in range(4):
        for k in ("ih", "hh"):
            s[f"dec_mi_layer.1.lstm.weight_{k}_l{l}"] = (2048, 512)
            s[f"dec_mi_layer.1.lstm.bias_{k}_l{l}"] = (2048,)
    for i in range(6):
        s[f"decoder.ups.{i}.0.weight"] = (VOC_UP_IN[i], VOC_UP_OUT[i], VOC_UP_KERNEL[i])
        s[f"decoder.ups.{i}.0.bias"] = (VOC_UP_OUT[i],)
    for rb in range(18):
        ch, K = VOC_UP_OUT[rb // 3], VOC_RB_KERNEL[rb % 3]
        p = f"decoder.resblocks.{rb}."
        for j in range(3):
            for c in ("convs1", "convs2"):
                s[p + f"{c}.{j}.weight"] = (ch, ch, K)
                s[p + f"{c}.{j}.bias"] = (ch,)
        for a in range(6):
            s[p + f"activations.{a}.act.alpha"] = (ch,)
            s[p + f"activations.{a}.act.beta"] = (ch,)
    s["decoder.activation_post.act.alpha"] = (24,)
    s["decoder.activation_post.act.beta"] = (24,)
    s["decoder.activation_post.upsample.filter"] = (24, 1, 12)
    s["decoder.activation_post.downsample.lowpass.filter"] = (24, 1, 12)
    s["decoder.conv_post.weight"] = (1, 24, 7)
    return s


def voc_weights(seed=5, aa_filter=None):
    """BigVGAN decoder weights scaled so that the signal stays of order one
    through all six stages and tanh stays mostly linear: convolutions
    N(0, g / sqrt(fan_in)) with g = 0.5 inside the AMP blocks and in conv_post,
    1 elsewhere, LSTM N(0, 0.5 / sqrt(512)), biases
    N(0, 0.02), log-scale snake alpha / beta N(0, 0.1).  The activation_post
    filters are `aa_filter` (12 taps) perturbed per channel by N(0, 1e-3)."""
    w = {}
    for name, shape in voc_shapes().items():
        if name.endswith(".bias") or "lstm.bias" in name:
            w[name] = normal(seed, name, shape, 0.02)
        elif name.endswith("act.alpha") or name.endswith("act.beta"):
            w[name] = normal(seed, name, shape, 0.1)
        elif name.endswith("filter"):
            base = np.zeros(12, np.float32) if aa_filter is None else np.asarray(aa_filter, np.float32)
            w[name] = (base[None, None, :] + normal(seed, name, shape, 1e-3)).astype(np.float32)
        elif "lstm.weight" in name:
            w[name] = normal(seed, name, shape, 0.5 / np.sqrt(512.0))
        elif "ups." in name:
            ic, oc, K = shape
            w[name] = normal(seed, name, shape, 1.0 / np.sqrt(2.0 * ic))
        else:
            fan_in = int(np.prod(shape[1:]))
            g = 0.5 if ("resblocks" in name or "conv_post" in name) else 1.0
            w[name] = normal(seed, name, shape, g / np.sqrt(fan_in))
    return w
