"""Seeded synthetic Qwen3-0.6B weights in the upstream ``load_weights`` format.

There is no network and no checkpoint on the build or benchmark hosts, so every
test and benchmark runs on random-init weights of the real architecture.  The
returned dict has exactly the keys and tensor layouts that the upstream
``load_weights`` builds (``Model/Qwen06B_architecture.py:163-170``):

* ``embed_weight``      fp16 [151936, 1024], tied to ``lm_head_weight``;
* ``layer_weights``     list of 11 fp16 tensors per layer, in the
  ``LDGLayerWeight`` field order (``Tools/megakernel/megakernel.cu:87-100``):
  input_layernorm, q_proj, k_proj, v_proj, q_norm, k_norm, o_proj,
  post_attention_layernorm, gate_proj, up_proj, down_proj, with the HF
  ``[out, in]`` row-major layout;
* ``final_norm_weight`` fp16 [1024];
* ``cos_table`` / ``sin_table`` fp16 [2048, 128], built as
  ``Model/Qwen06B_architecture.py:134-142`` does (fp32 ``inv_freq`` with
  theta 1e6, ``outer`` with fp32 positions, cos/sin, ``repeat(1, 2)``, fp16).

Generation order is fixed: one ``torch.Generator('cpu').manual_seed(seed)``;
the embedding first, then per layer every matrix in table order, each drawn in
fp32 from N(0, std) and cast to fp16.  All RMSNorm weights are 1.0.  Because
the embedding and the layers are drawn in order, the first ``n`` layers of a
28-layer draw equal an ``n``-layer draw with the same seed.
"""
from __future__ import annotations

import torch

NUM_LAYERS = 28
HIDDEN_SIZE = 1024
INTERMEDIATE_SIZE = 3072
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
Q_SIZE = NUM_Q_HEADS * HEAD_DIM
KV_SIZE = NUM_KV_HEADS * HEAD_DIM
VOCAB_SIZE = 151936
MAX_SEQ_LEN = 2048
ROPE_THETA = 1_000_000.0
RMS_EPS = 1e-6

# (name, shape) in LDGLayerWeight order; shape None marks an RMSNorm weight.
LAYER_FIELDS = (
    ("input_layernorm", (HIDDEN_SIZE,)),
    ("q_proj", (Q_SIZE, HIDDEN_SIZE)),
    ("k_proj", (KV_SIZE, HIDDEN_SIZE)),
    ("v_proj", (KV_SIZE, HIDDEN_SIZE)),
    ("q_norm", (HEAD_DIM,)),
    ("k_norm", (HEAD_DIM,)),
    ("o_proj", (HIDDEN_SIZE, Q_SIZE)),
    ("post_attention_layernorm", (HIDDEN_SIZE,)),
    ("gate_proj", (INTERMEDIATE_SIZE, HIDDEN_SIZE)),
    ("up_proj", (INTERMEDIATE_SIZE, HIDDEN_SIZE)),
    ("down_proj", (HIDDEN_SIZE, INTERMEDIATE_SIZE)),
)


def rope_tables(max_seq_len: int = MAX_SEQ_LEN, theta: float = ROPE_THETA,
                head_dim: int = HEAD_DIM) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 cos/sin tables [max_seq_len, head_dim] (rotate-half convention)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    positions = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(positions, inv_freq)
    cos = torch.cos(freqs).repeat(1, 2).to(torch.float16).contiguous()
    sin = torch.sin(freqs).repeat(1, 2).to(torch.float16).contiguous()
    return cos, sin


def _normal(gen: torch.Generator, shape, std: float) -> torch.Tensor:
    t = torch.empty(shape, dtype=torch.float32)
    t.normal_(0.0, std, generator=gen)
    return t.to(torch.float16)


def synthetic_weights(seed: int = 0, num_layers: int = NUM_LAYERS, std: float = 0.02,
                      device: str | torch.device = "cpu",
                      max_seq_len: int = MAX_SEQ_LEN) -> dict:
    """Random-init weights dict with the upstream ``load_weights`` layout."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed))
    embed = _normal(gen, (VOCAB_SIZE, HIDDEN_SIZE), std)
    layers: list[torch.Tensor] = []
    for _ in range(num_layers):
        for _name, shape in LAYER_FIELDS:
            if len(shape) == 1:
                layers.append(torch.ones(shape, dtype=torch.float16))
            else:
                layers.append(_normal(gen, shape, std))
    final_norm = torch.ones(HIDDEN_SIZE, dtype=torch.float16)
    cos, sin = rope_tables(max_seq_len)
    out = dict(
        embed_weight=embed,
        layer_weights=layers,
        final_norm_weight=final_norm,
        cos_table=cos,
        sin_table=sin,
    )
    if str(device) != "cpu":
        out = {k: ([t.to(device) for t in v] if isinstance(v, list) else v.to(device))
               for k, v in out.items()}
    out["lm_head_weight"] = out["embed_weight"]
    return out


def hf_state_dict(weights: dict) -> dict:
    """Map a weights dict to HF ``Qwen3ForCausalLM`` state-dict names (fp32)."""
    sd = {"model.embed_tokens.weight": weights["embed_weight"].float(),
          "model.norm.weight": weights["final_norm_weight"].float(),
          "lm_head.weight": weights["lm_head_weight"].float()}
    lw = weights["layer_weights"]
    names = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
             "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
             "self_attn.o_proj.weight", "post_attention_layernorm.weight",
             "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
    for li in range(len(lw) // 11):
        for j, n in enumerate(names):
            sd[f"model.layers.{li}.{n}"] = lw[li * 11 + j].float()
    return sd
