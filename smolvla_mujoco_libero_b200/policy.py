"""Drop-in ``sample_actions`` for SmolVLA policies.

``SampleActions`` mirrors the reference's deployment boundary
(deploy/trt_sample_actions_core_deploy.py:259-310): it is installed by assignment over
``policy.model.sample_actions`` and takes the same arguments,

    sample_actions(images, img_masks, lang_tokens, lang_masks, state, noise=None, **kwargs)

images: list of fp32 [B, 3, 512, 512]; img_masks: list of bool [B]; lang_tokens int64 [B, T] and lang_masks
bool [B, T] (padded / truncated to the configured length like match_static_shape, :276-286); state [B, <=32]
(zero-padded); noise [B, 50, 32] or None (then drawn N(0,1)).  Returns fp32 [B, chunk, action_dim].
Unlike the reference's static engine (batch 1 only, :290-291) any batch size works: one runner (static
buffers + CUDA graph) is built and captured per batch size on first use.
"""

from __future__ import annotations

from typing import Any

import torch

from .config import SmolVLAConfig
from .model import DeviceWeights, SmolVLARunner


class SampleActions:
    def __init__(self, cfg: SmolVLAConfig, weights: DeviceWeights, use_cuda_graph: bool = True,
                 action_dim: int | None = None, split_k: bool = True, flow: bool | None = None):
        if not weights.quantized:
            raise ValueError("SampleActions needs weights packed with a scale table")
        self.cfg, self.weights, self.use_cuda_graph, self.split_k = cfg, weights, use_cuda_graph, split_k
        # flow: the persistent flow-matching kernel for batch * chunk <= 64 rows (None = wherever it applies)
        self.flow = flow
        self.action_dim = cfg.action_dim if action_dim is None else action_dim
        self.runners: dict[int, SmolVLARunner] = {}
        self.stats: dict[str, Any] = {"cuda_graph_failed": False}

    def runner(self, batch: int) -> SmolVLARunner:
        r = self.runners.get(batch)
        if r is None:
            # flow=True asks for the kernel wherever it applies (large batches keep the per-layer launches)
            r = SmolVLARunner(self.weights, batch, split_k=self.split_k, flow=False if self.flow is False else None)
            if self.use_cuda_graph:
                try:
                    r.capture()
                except RuntimeError as exc:  # capture refused: run the launch list directly
                    r.graph = None
                    self.stats["cuda_graph_failed"] = True
                    self.stats["cuda_graph_error"] = str(exc)
            self.runners[batch] = r
        return r

    @torch.no_grad()
    def __call__(self, images, img_masks, lang_tokens, lang_masks, state, noise=None, **_kwargs) -> torch.Tensor:
        c = self.cfg
        bsize = state.shape[0]
        dev = self.weights.device
        if noise is None:
            noise = torch.randn(bsize, c.chunk, c.max_action_dim, dtype=torch.float32, device=dev)
        r = self.runner(bsize)
        out = r(images, img_masks, lang_tokens, lang_masks, state, noise)
        return out[:, :, : self.action_dim].clone()


class PrefixFeatures:
    """The RL-token consumer's features: the prefix prefill of ``sample_actions`` alone, keeping the
    final-layer prefix hidden states (``RLTokenExtractor.extract``, smollvla_rltoken/rlt/rl_token.py:50-88).

    ``extract`` returns ``z`` fp32 [B, Lp, hidden] (the final RMSNorm of the last text layer's output, as the
    reference's ``outputs_embeds[0]``), ``pad_mask`` bool [B, Lp], ``n_img_tokens`` and ``kv_cache``: per text
    layer the (K post-RoPE, V) bf16 tensors [B, Lp, kv_heads * 64] that the action expert reads.  The same
    quantized kernels as ``SampleActions``; one CUDA graph per batch size."""

    def __init__(self, cfg: SmolVLAConfig, weights: DeviceWeights, use_cuda_graph: bool = True):
        if not weights.quantized:
            raise ValueError("PrefixFeatures needs weights packed with a scale table")
        self.cfg, self.weights, self.use_cuda_graph = cfg, weights, use_cuda_graph
        self.runners: dict[int, SmolVLARunner] = {}

    def runner(self, batch: int) -> SmolVLARunner:
        r = self.runners.get(batch)
        if r is None:
            r = SmolVLARunner(self.weights, batch, prefix_only=True)
            if self.use_cuda_graph:
                r.capture()
            self.runners[batch] = r
        return r

    @torch.no_grad()
    def extract(self, images, img_masks, lang_tokens, lang_masks, state) -> dict[str, Any]:
        c = self.cfg
        B = state.shape[0]
        r = self.runner(B)
        r.load_inputs(images, img_masks, lang_tokens, lang_masks, state, None)
        r.run()
        Lp = c.prefix_len
        return {
            "z": r.prefix_out.view(B, Lp, c.hidden).float(),
            "pad_mask": r.key_pad.bool().clone(),
            "n_img_tokens": c.n_cams * c.n_img_tokens,
            "kv_cache": [(r.kcache[i].view(B, Lp, -1).clone(), r.vcache[i].view(B, Lp, -1).clone())
                         for i in range(c.text_layers)],
        }


def install_sample_actions(policy: Any, sample_actions: SampleActions) -> dict[str, Any]:
    """Replace ``policy.model.sample_actions`` (the reference installs its TensorRT runner the same way,
    deploy/trt_sample_actions_core_deploy.py:310)."""
    policy.model.sample_actions = sample_actions
    return {"backend": "svla-b200", "replacement": "policy.model.sample_actions core",
            "cuda_graph": sample_actions.use_cuda_graph}
