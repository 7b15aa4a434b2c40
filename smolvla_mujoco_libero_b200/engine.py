"""The whole sample_actions call in native code: a thin ctypes handle over ``svla_engine_*`` (include/svla.h).

``NativeSampleActions`` takes the reference's arguments, like ``SampleActions``
(deploy/trt_sample_actions_core_deploy.py:259-310), but the launch list, its buffers and its CUDA graphs
live in libsvla.so: Python only passes pointers.  The engine loads a packed-weights file written by
``checkpoint.save_packed``; for the same file and inputs its actions are bit-identical to
``SmolVLARunner``'s (same kernels, same descriptors, same order).

Inputs may be CUDA tensors or CPU tensors (pinned or pageable); the engine copies them on the current
stream.  Pinned host inputs must stay alive until the stream has consumed them.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any

import torch

from . import _lib as L
from ._lib import check, lib


def _info_dict(info: L.EngineInfo) -> dict[str, int]:
    return {name: int(getattr(info, name)) for name, _ in L.EngineInfo._fields_}


def inspect(path: str | Path) -> dict[str, int]:
    """Dimensions and sizes of a packed-weights file (parsed and validated on the host, no GPU needed)."""
    info = L.EngineInfo()
    check(lib().svla_engine_inspect(str(path).encode(), ctypes.byref(info)), "svla_engine_inspect")
    return _info_dict(info)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class NativeSampleActions:
    """``sample_actions(images, img_masks, lang_tokens, lang_masks, state, noise=None)`` through the native
    engine, for up to ``max_batch`` samples per call."""

    def __init__(self, packed_path: str | Path, max_batch: int = 1, use_cuda_graph: bool = True,
                 split_k: bool = True, device: str | torch.device = "cuda", action_dim: int | None = None,
                 flow: bool = True):
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        flags = (0 if use_cuda_graph else L.ENGINE_NO_GRAPH) | (0 if split_k else L.ENGINE_NO_SPLIT_K) | \
            (0 if flow else L.ENGINE_NO_FLOW)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().svla_engine_create(str(packed_path).encode(), int(max_batch), flags, _stream(self.device),
                                           ctypes.byref(handle)), "svla_engine_create")
        self._h = handle
        self.info = self._get_info()
        self.action_dim = self.info["action_dim"] if action_dim is None else action_dim

    def _get_info(self) -> dict[str, int]:
        info = L.EngineInfo()
        check(lib().svla_engine_get_info(self._h, ctypes.byref(info)), "svla_engine_get_info")
        return _info_dict(info)

    @property
    def launches_per_call(self) -> int:
        return self.info["launches_per_call"]

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().svla_engine_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may already be gone
            pass

    @staticmethod
    def _arg(t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
        if t.dtype == torch.bool and dtype == torch.uint8:
            t = t.contiguous().view(torch.uint8)
        if t.dtype != dtype:
            raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        return t

    @torch.no_grad()
    def sample_actions(self, images, img_masks, lang_tokens, lang_masks, state, noise=None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Actions fp32 [B, chunk, max_action_dim] (into ``out`` when given: a CUDA or CPU tensor)."""
        if self._h is None:
            raise RuntimeError("engine is closed")
        i = self.info
        bsize = int(state.shape[0])
        if len(images) != i["n_cams"] or len(img_masks) != i["n_cams"]:
            raise ValueError(f"expected {i['n_cams']} cameras")
        if noise is None:
            noise = torch.randn(bsize, i["chunk"], i["max_action_dim"], dtype=torch.float32, device=self.device)
        imgs = [self._arg(x, torch.float32, "images") for x in images]
        masks = [self._arg(m, torch.uint8, "img_masks") for m in img_masks]
        tokens = self._arg(lang_tokens, torch.int64, "lang_tokens")
        lmask = self._arg(lang_masks, torch.uint8, "lang_masks")
        st = self._arg(state, torch.float32, "state")
        nz = self._arg(noise, torch.float32, "noise")
        shape = (bsize, i["chunk"], i["max_action_dim"])
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=self.device)
        elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"out must be contiguous fp32 {shape}")
        n = i["n_cams"]
        img_p = (ctypes.c_void_p * n)(*[x.data_ptr() for x in imgs])
        mask_p = (ctypes.c_void_p * n)(*[m.data_ptr() for m in masks])
        with torch.cuda.device(self.device):
            check(lib().svla_engine_sample_actions(
                self._h, img_p, mask_p, tokens.data_ptr(), lmask.data_ptr(), int(tokens.shape[1]), st.data_ptr(),
                int(st.shape[1]), nz.data_ptr(), bsize, out.data_ptr(), _stream(self.device)),
                "svla_engine_sample_actions")
        return out

    def __call__(self, images, img_masks, lang_tokens, lang_masks, state, noise=None, **_kwargs: Any) -> torch.Tensor:
        """The reference's return: fp32 [B, chunk, action_dim]."""
        return self.sample_actions(images, img_masks, lang_tokens, lang_masks, state, noise)[:, :, :self.action_dim]
