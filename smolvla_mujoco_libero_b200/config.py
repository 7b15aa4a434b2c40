"""SmolVLA sample_actions configuration.

Defaults are the benchmark architecture: SigLIP 12 x 768 (patch 16, 512 px), pixel shuffle x4 to 64 tokens per
image, SmolVLM2 text 16 x 960 (15 q / 5 kv heads, head_dim 64, MLP 2560), action expert 16 x 720 (MLP 2048,
self-attention on even layers, cross-attention to the prefix KV on odd layers), 48 language tokens, state
and actions padded to 32, chunk 50, 10 Euler flow-matching steps.

Every count and width is a field; nothing in the kernels or the runner bakes them in.  The RoPE wavelength
defaults to 10 000, the value the reference's attention uses (lerobot apply_rope(..., max_wavelength=10_000),
deploy/validate_fused_rope_layout_math.py:28); SmolVLM2's text config states 100 000.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class SmolVLAConfig:
    # vision tower (SigLIP) and connector
    image_size: int = 512
    patch: int = 16
    channels: int = 3
    vis_hidden: int = 768
    vis_layers: int = 12
    vis_heads: int = 12
    vis_mlp: int = 3072
    vis_eps: float = 1e-6
    scale_factor: int = 4
    n_cams: int = 2
    # SmolVLM2 text model
    hidden: int = 960
    text_layers: int = 16
    heads: int = 15
    kv_heads: int = 5
    head_dim: int = 64
    mlp: int = 2560
    rms_eps: float = 1e-5
    vocab: int = 49280
    rope_wavelength: float = 10_000.0
    # action expert
    expert_hidden: int = 720
    expert_layers: int = 16
    expert_mlp: int = 2048
    self_attn_every_n_layers: int = 2
    # policy
    n_lang: int = 48
    max_state_dim: int = 32
    max_action_dim: int = 32
    action_dim: int = 7
    chunk: int = 50
    num_steps: int = 10
    min_period: float = 4e-3
    max_period: float = 4.0
    # SmoothQuant recipe (deploy/5Osmoothquant-alpha085-full-w8a8-deploy-eval.sh:19-20)
    alpha: float = 0.85
    percentile: float = 99.99

    @property
    def grid(self) -> int:
        return self.image_size // self.patch

    @property
    def n_patches(self) -> int:
        return self.grid * self.grid

    @property
    def n_img_tokens(self) -> int:
        return self.n_patches // (self.scale_factor ** 2)

    @property
    def prefix_len(self) -> int:
        return self.n_cams * self.n_img_tokens + self.n_lang + 1

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    def is_cross_layer(self, layer: int) -> bool:
        """lerobot SmolVLMWithExpertModel.forward: cross-attention unless layer % n == 0."""
        return not (self.self_attn_every_n_layers > 0 and layer % self.self_attn_every_n_layers == 0)

    def as_dict(self) -> dict:
        return asdict(self)

    def with_(self, **kw) -> "SmolVLAConfig":
        return replace(self, **kw)


BENCH = SmolVLAConfig()

# A small configuration with the same structure, for fast parity tests of the whole path.
TINY = SmolVLAConfig(image_size=128, vis_layers=2, text_layers=4, expert_layers=4, n_lang=16, num_steps=3)

# Module-name prefixes of the reference checkpoint (regexes at
# deploy/5Osmoothquant-alpha085-full-w8a8-deploy-eval.sh:40-42).
TEXT = "model.vlm_with_expert.vlm.model.text_model"
EXPERT = "model.vlm_with_expert.lm_expert"
VISION = "model.vlm_with_expert.vlm.model.vision_model"
CONNECTOR = "model.vlm_with_expert.vlm.model.connector.modality_projection.proj"
