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

from collections import OrderedDict
from typing import Any

import torch

from .config import SmolVLAConfig
from .model import DeviceWeights, SmolVLARunner


def debug_output_names(cfg: SmolVLAConfig) -> list[str]:
    """Output names of the reference's debug core, in its order (deploy/diagnose_3_4_numeric_baseline.py:66-70)."""
    names = ["action_chunk", "prefix_embs", "prefix_out"]
    for step in range(cfg.num_steps):
        names += [f"suffix_out_step_{step:02d}", f"v_t_step_{step:02d}", f"x_t_step_{step:02d}"]
    return names


class SampleActions:
    def __init__(self, cfg: SmolVLAConfig, weights: DeviceWeights, use_cuda_graph: bool = True,
                 action_dim: int | None = None, split_k: bool = True, flow: bool | None = None):
        if not weights.quantized:
            raise ValueError("SampleActions needs weights packed with a scale table")
        self.cfg, self.weights, self.use_cuda_graph, self.split_k = cfg, weights, use_cuda_graph, split_k
        # flow: the persistent flow-matching kernel for batch * chunk <= 64 rows (None = wherever it applies)
        self.flow = flow
        self.action_dim = cfg.action_dim if action_dim is None else action_dim
        self.runners: dict[tuple[int, bool, bool], SmolVLARunner] = {}
        self.stats: dict[str, Any] = {"cuda_graph_failed": False}

    def runner(self, batch: int, image_embeds: bool = False, debug: bool = False) -> SmolVLARunner:
        """The runner for one batch size and input mode, built (and captured as a CUDA graph) on first use.
        Debug runners run their launches one by one so that the taps see every intermediate in stream order."""
        key = (batch, bool(image_embeds), bool(debug))
        r = self.runners.get(key)
        if r is None:
            # flow=True asks for the kernel wherever it applies (large batches keep the per-layer launches)
            r = SmolVLARunner(self.weights, batch, split_k=self.split_k, debug_taps=debug,
                              flow=False if (self.flow is False or debug) else None, image_embeds=image_embeds)
            if self.use_cuda_graph and not debug:
                try:
                    r.capture()
                except RuntimeError as exc:  # capture refused: run the launch list directly
                    r.graph = None
                    self.stats["cuda_graph_failed"] = True
                    self.stats["cuda_graph_error"] = str(exc)
            self.runners[key] = r
        return r

    def _noise(self, bsize: int, noise):
        if noise is not None:
            return noise
        c = self.cfg
        return torch.randn(bsize, c.chunk, c.max_action_dim, dtype=torch.float32, device=self.weights.device)

    @torch.no_grad()
    def __call__(self, images, img_masks, lang_tokens, lang_masks, state, noise=None, **_kwargs) -> torch.Tensor:
        bsize = state.shape[0]
        r = self.runner(bsize)
        out = r(images, img_masks, lang_tokens, lang_masks, state, self._noise(bsize, noise))
        return out[:, :, : self.action_dim].clone()

    @torch.no_grad()
    def from_image_embeds(self, image_embs, img_masks, lang_tokens, lang_masks, state, noise=None) -> torch.Tensor:
        """Embeds mode of the exported core (deploy/export_smolvla_sample_actions_onnx.py:64-164): one bf16
        [B, n_img_tokens, hidden] image embedding per camera (the connector's output) replaces the images."""
        bsize = state.shape[0]
        r = self.runner(bsize, image_embeds=True)
        out = r(image_embs, img_masks, lang_tokens, lang_masks, state, self._noise(bsize, noise))
        return out[:, :, : self.action_dim].clone()

    @torch.no_grad()
    def debug_outputs(self, images, img_masks, lang_tokens, lang_masks, state, noise=None,
                      image_embeds: bool = False) -> "OrderedDict[str, torch.Tensor]":
        """The reference's debug core (SmolVLADebugCoreWrapper, deploy/diagnose_3_4_numeric_baseline.py:47-206):
        action_chunk [B, chunk, action_dim]; prefix_embs and prefix_out [B, Lp, hidden]; per flow step
        suffix_out_step_NN [B, chunk, expert_hidden] (the expert output action_out_proj reads),
        v_t_step_NN and x_t_step_NN [B, chunk, max_action_dim] (fp32).  Runs the same kernels as the
        deployed call, launched one by one, with the fused-away intermediates also written out."""
        c = self.cfg
        bsize = state.shape[0]
        r = self.runner(bsize, image_embeds=image_embeds, debug=True)
        wanted = set(debug_output_names(c))
        taps: dict[str, torch.Tensor] = {}

        def observe(names, buf):
            for n in names:
                if n in wanted:
                    taps[n] = buf.clone()

        r.load_inputs(images, img_masks, lang_tokens, lang_masks, state, self._noise(bsize, noise))
        r.run(observer=observe)
        out: OrderedDict[str, torch.Tensor] = OrderedDict()
        out["action_chunk"] = r.actions()[:, :, : self.action_dim].clone()
        shapes = {"prefix_embs": (bsize, c.prefix_len, c.hidden), "prefix_out": (bsize, c.prefix_len, c.hidden)}
        for name in debug_output_names(c)[1:]:
            shape = shapes.get(name)
            if shape is None:
                width = c.expert_hidden if name.startswith("suffix_out") else c.max_action_dim
                shape = (bsize, c.chunk, width)
            out[name] = taps[name].view(shape)
        return out


class SampleActionsCore:
    """Tensor-only core with the exported signature, images mode (deploy/export_smolvla_sample_actions_onnx.py:
    28-61): (image, image2, image_mask, image2_mask, state, language_tokens, language_attention_mask, noise) ->
    action_chunk [B, chunk, action_dim]; inputs already pre-processed (resized, normalised, padded)."""

    input_names = ["image", "image2", "image_mask", "image2_mask", "state", "language_tokens",
                   "language_attention_mask", "noise"]

    def __init__(self, sample_actions: SampleActions):
        self.sa = sample_actions

    def __call__(self, image, image2, image_mask, image2_mask, state, language_tokens, language_attention_mask,
                 noise):
        return self.sa([image, image2], [image_mask, image2_mask], language_tokens, language_attention_mask, state,
                       noise)


class SampleActionsFromEmbedsCore(SampleActionsCore):
    """Embeds mode of the exported core (deploy/export_smolvla_sample_actions_onnx.py:64-164, input names :340-349):
    image_emb / image2_emb bf16 [B, n_img_tokens, hidden] instead of the images."""

    input_names = ["image_emb", "image2_emb", "image_mask", "image2_mask", "state", "language_tokens",
                   "language_attention_mask", "noise"]

    def __call__(self, image_emb, image2_emb, image_mask, image2_mask, state, language_tokens,
                 language_attention_mask, noise):
        return self.sa.from_image_embeds([image_emb, image2_emb], [image_mask, image2_mask], language_tokens,
                                         language_attention_mask, state, noise)


class DebugCore(SampleActionsFromEmbedsCore):
    """SmolVLADebugCoreWrapper's contract (deploy/diagnose_3_4_numeric_baseline.py:47-206): the embeds-mode core
    returning the tuple named by ``output_names`` (action_chunk, prefix_embs, prefix_out, then suffix_out /
    v_t / x_t for every flow step).  ``image_embeds=False`` takes the images instead."""

    def __init__(self, sample_actions: SampleActions, image_embeds: bool = True):
        super().__init__(sample_actions)
        self.image_embeds = image_embeds
        self.output_names = debug_output_names(sample_actions.cfg)

    def __call__(self, image_emb, image2_emb, image_mask, image2_mask, state, language_tokens,
                 language_attention_mask, noise):
        outs = self.sa.debug_outputs([image_emb, image2_emb], [image_mask, image2_mask], language_tokens,
                                     language_attention_mask, state, noise, image_embeds=self.image_embeds)
        return tuple(outs[n] for n in self.output_names)


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
