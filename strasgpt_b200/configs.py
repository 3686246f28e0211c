"""Model configurations: the five benchmark shapes and small test shapes.

Each entry fixes every hyperparameter the forward pass reads (the keys
source/json_parser.y:81-189 of the reference picks out of config.json) plus
the workload (prompt length P and greedy decode steps S). Values the
benchmark description leaves open are pinned here once:
  - rms_norm_eps: 1e-5 (Llama, Mistral, MoE), 1e-6 (Qwen3);
  - MoE rope_theta 150000, untied LM head, low nibble = even element;
  - max_position_embeddings = P + S rounded up to 64;
  - weights N(0, 0.02) in bf16, RMSNorm gains 1.0, MXFP4 codes uniform over
    the 16 values and e8m0 scale bytes uniform in [119, 127] (2^-8 .. 2^0);
  - prompt ids: numpy.random.default_rng(seed).integers(0, V, P).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass


@dataclass(frozen=True)
class ModelConfig:
    name: str
    model_type: str
    dim: int            # hidden_size (D)
    hidden: int         # intermediate_size (F); expert FFN size for MoE
    layers: int         # num_hidden_layers (L)
    q_heads: int        # num_attention_heads (QH)
    kv_heads: int       # num_key_value_heads (KH)
    head_dim: int       # HD
    vocab: int          # V
    rope_theta: float
    eps: float
    tied: bool          # LM head aliased to the embedding
    qk_norm: bool = False
    rope_interleaved: bool = False
    experts: int = 0    # num_local_experts (0: dense)
    top_k: int = 0      # num_experts_per_tok
    prompt_len: int = 8
    steps: int = 16
    bos_token_id: int = 1
    eos_token_id: int = 2

    @property
    def context_len(self) -> int:
        n = self.prompt_len + self.steps
        return (n + 63) // 64 * 64

    def with_(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    # Algorithmic bytes one decode token streams on ONE gpu holding the whole
    # model: every weight once (the active experts only for MoE) plus the
    # KV cache read at context position `pos` (fp32) and the new K/V row.
    def decode_weight_bytes(self) -> int:
        D, F, L = self.dim, self.hidden, self.layers
        qd, kd = self.q_heads * self.head_dim, self.kv_heads * self.head_dim
        per_layer = (qd + 2 * kd) * D * 2 + D * qd * 2 + 2 * D * 2
        if self.qk_norm:
            per_layer += 2 * self.head_dim * 2
        if self.experts:
            per_layer += self.experts * D * 2  # router
            blocks = lambda rows, k: rows * (k // 32) * 17  # 16 B codes + scale
            per_layer += self.top_k * (2 * blocks(F, D) + blocks(D, F))
        else:
            per_layer += 3 * D * F * 2
        lm_head = self.vocab * D * 2
        return L * per_layer + lm_head + D * 2

    def kv_bytes(self, pos: int) -> int:
        # read K and V rows [0, pos] and write row pos, fp32
        row = 2 * self.layers * self.kv_heads * self.head_dim * 4
        return row * (pos + 1) + row

    def prefill_flops_per_token(self) -> float:
        D, F, L = self.dim, self.hidden, self.layers
        qd, kd = self.q_heads * self.head_dim, self.kv_heads * self.head_dim
        per_layer = (qd + 2 * kd) * D + D * qd
        if self.experts:
            per_layer += self.experts * D + self.top_k * 3 * D * F
        else:
            per_layer += 3 * D * F
        return 2.0 * L * per_layer


# The five benchmark configurations.
C1 = ModelConfig("c1_llama1b", "llama", 2048, 8192, 16, 32, 8, 64, 128256,
                 500000.0, 1e-5, tied=True, prompt_len=8, steps=16,
                 bos_token_id=128000, eos_token_id=128001)
C2 = ModelConfig("c2_qwen3_0p6b", "qwen3", 1024, 3072, 28, 16, 8, 128, 151936,
                 1000000.0, 1e-6, tied=True, qk_norm=True, prompt_len=512,
                 steps=128, bos_token_id=151643, eos_token_id=151645)
C3 = ModelConfig("c3_llama8b", "llama", 4096, 14336, 32, 32, 8, 128, 128256,
                 500000.0, 1e-5, tied=False, prompt_len=2048, steps=256,
                 bos_token_id=128000, eos_token_id=128001)
C4 = ModelConfig("c4_moe_mxfp4", "strasgpt_moe", 2880, 2880, 24, 64, 8, 64,
                 201088, 150000.0, 1e-5, tied=False, experts=32, top_k=4,
                 prompt_len=1024, steps=128, bos_token_id=199998,
                 eos_token_id=200002)
C5 = ModelConfig("c5_mistral24b", "mistral", 5120, 32768, 40, 32, 8, 128,
                 131072, 100000000.0, 1e-5, tied=False, prompt_len=8192,
                 steps=256, bos_token_id=1, eos_token_id=2)

BENCH = {c.name: c for c in (C1, C2, C3, C4, C5)}

# C5's width (D 5120, F 32768, 32/8 heads, theta 1e8, untied) and its full
# 8192-token prompt on 4 layers: the long-context paths (8448-row KV
# attention, multi-chunk prefill) at a CPU cost the reference finishes in
# minutes, for a full-logits parity fixture.
C5_L4 = C5.with_(name="c5_mistral24b_l4", layers=4, steps=64)

PARITY = {c.name: c for c in (C5_L4,)}

# C3's layer shapes on 2 layers with a 32768-row LM head and a 64-token
# prompt: the small case (about 1.4 GB on the device) on which the decode
# kernel is captured under ncu; its DRAM traffic over algorithmic bytes
# carries over to C3, whose layers are identical.
C3_S = C3.with_(name="c3s_llama8b_l2", layers=2, vocab=32768, prompt_len=64,
                steps=8, bos_token_id=1, eos_token_id=2)
# The same 2-layer model with C3's 2048-token prompt: the prefill kernels
# (projections, attention) at C3's shapes, captured under ncu with a few GB
# on the device.
C3_P = C3_S.with_(name="c3p_llama8b_l2", prompt_len=2048, steps=4)

PROFILE = {c.name: c for c in (C3_S, C3_P)}

# Small shapes with the same structural features, for fast parity tests.
T_LLAMA = ModelConfig("t_llama", "llama", 256, 512, 2, 8, 2, 32, 1024,
                      500000.0, 1e-5, tied=True, prompt_len=8, steps=8)
T_QWEN = ModelConfig("t_qwen", "qwen3", 256, 384, 2, 4, 2, 64, 1024,
                     1000000.0, 1e-6, tied=True, qk_norm=True, prompt_len=24,
                     steps=8)
T_UNTIED = ModelConfig("t_untied", "llama", 512, 1024, 2, 8, 2, 64, 2048,
                       500000.0, 1e-5, tied=False, prompt_len=16, steps=8)
T_GQA8 = ModelConfig("t_gqa8", "mistral", 256, 512, 2, 16, 2, 64, 1024,
                     100000000.0, 1e-5, tied=False, prompt_len=40, steps=8)
T_INTERLEAVED = ModelConfig("t_interleaved", "qwen3", 256, 512, 2, 4, 2, 64,
                            1024, 1000000.0, 1e-6, tied=True, qk_norm=True,
                            rope_interleaved=True, prompt_len=12, steps=6)
T_CHUNK = ModelConfig("t_chunk", "llama", 128, 256, 2, 4, 2, 32, 512,
                      500000.0, 1e-5, tied=True, prompt_len=600, steps=4)
T_MOE = ModelConfig("t_moe", "strasgpt_moe", 256, 256, 2, 8, 2, 32, 1024,
                    150000.0, 1e-5, tied=False, experts=8, top_k=4,
                    prompt_len=12, steps=8)

TINY = {c.name: c for c in (T_LLAMA, T_QWEN, T_UNTIED, T_GQA8, T_INTERLEAVED,
                            T_CHUNK, T_MOE)}

ALL = {**BENCH, **PARITY, **PROFILE, **TINY}


def get(name: str) -> ModelConfig:
    try:
        return ALL[name]
    except KeyError:
        raise KeyError(f"unknown config {name!r}; known: {sorted(ALL)}")
