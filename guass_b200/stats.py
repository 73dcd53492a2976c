"""Densify statistics in one launch per step.

GUASS's ``GaussianStatsTracker`` (gaussian_peft/controllers/stats.py:18-109)
runs after every backward (trainers/base_trainer.py:61) and costs about ten
tensor operations per Gaussian layer: 128 layers make well over a thousand
small launches per step.  :class:`BatchedStatsTracker` has the same methods
and returns the same scores, but a step's update for every layer is one
``gf_grad_stats_accumulate`` launch.

Per Gaussian k of a layer (stats.py:47-66, 116-131):
  grad_mu += ||mu_raw.grad[k]||_2      grad_cov += ||chol_raw.grad[k]||_2
  grad_amp += |amp.grad[k]|            contrib  += |amp[k]|
  active_steps += 1
Each layer's five accumulators are the rows of one ``[5, K]`` fp32 tensor;
``get_scores`` returns ``[K, 1]`` views like the reference.
"""
from __future__ import annotations

import torch

from guass_b200 import _lib

_PLANES = ("grad_mu", "grad_cov", "grad_amp", "contrib", "active_steps")


class BatchedStatsTracker:
    """Same interface as gaussian_peft.controllers.stats.GaussianStatsTracker
    (fp32 accumulators on a CUDA device)."""

    def __init__(self) -> None:
        self._layers: dict[str, torch.Tensor] = {}

    def register_layer(self, layer_name: str, num_gaussians: int, device, dtype: torch.dtype = torch.float32) -> None:
        if dtype != torch.float32:
            raise ValueError("BatchedStatsTracker accumulates in float32")
        dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError(f"BatchedStatsTracker needs a CUDA device, got {dev}")
        self._layers[layer_name] = torch.zeros(len(_PLANES), int(num_gaussians), device=dev, dtype=torch.float32)

    def ensure_layer(self, layer_name: str, num_gaussians: int, device, dtype: torch.dtype = torch.float32) -> None:
        stats = self._layers.get(layer_name)
        if stats is None or stats.shape[1] != num_gaussians:
            self.register_layer(layer_name, num_gaussians, device, dtype=dtype)

    # -- updates -------------------------------------------------------------
    @staticmethod
    def _operand(t, k: int, cols: int, stats: torch.Tensor, keep: list):
        if t is None:
            return None
        t = t.detach()
        if t.numel() != k * cols:
            raise RuntimeError(f"expected {k}x{cols} values, got shape {tuple(t.shape)}")
        if t.device != stats.device:
            raise RuntimeError(f"tensor on {t.device}, statistics on {stats.device}")
        if t.dtype != torch.float32 or not t.is_contiguous():
            t = t.to(torch.float32).contiguous()
        keep.append(t)
        return t.data_ptr()

    def _launch(self, entries) -> None:
        """entries: (layer_name, mu_grad, chol_grad, amp_grad, amp_value).
        Operands that need a dtype conversion are converted on the current
        stream, the launch's stream, so their memory is not reused before
        the kernel has read them."""
        L = _lib.lib()
        stream = torch.cuda.current_stream(self._layers[entries[0][0]].device)
        for start in range(0, len(entries), _lib.GF_MAX_FIELDS):
            chunk = entries[start:start + _lib.GF_MAX_FIELDS]
            arr = (_lib.GfStatsLayer * len(chunk))()
            keep = []
            for d, (name, mu_g, chol_g, amp_g, amp_v) in zip(arr, chunk):
                stats = self._layers[name]
                k = stats.shape[1]
                d.num_gaussians = k
                d.d_mu_raw = self._operand(mu_g, k, 2, stats, keep)
                d.d_chol_raw = self._operand(chol_g, k, 3, stats, keep)
                d.d_amp = self._operand(amp_g, k, 1, stats, keep)
                d.amp = self._operand(amp_v, k, 1, stats, keep)
                d.stats = stats.data_ptr()
            _lib.check(L.gf_grad_stats_accumulate(len(chunk), arr, stream.cuda_stream))

    def update_from_layer_grads(self, layer_name: str, mu_grad, chol_grad, amp_grad, amp_value=None) -> None:
        self._launch([(layer_name, mu_grad, chol_grad, amp_grad, amp_value)])

    def update_from_model(self, model) -> None:
        entries = []
        for module_name, module in model.named_modules():
            if not all(hasattr(module, n) for n in ("mu_raw", "chol_raw", "amp")):
                continue
            self.ensure_layer(module_name, int(module.mu_raw.shape[0]), module.mu_raw.device)
            entries.append((module_name, module.mu_raw.grad, module.chol_raw.grad, module.amp.grad,
                            module.amp.detach()))
        if entries:
            self._launch(entries)

    # -- reads ---------------------------------------------------------------
    def get_scores(self, layer_name: str) -> dict[str, torch.Tensor]:
        s = self._layers[layer_name]
        col = {n: s[i].view(-1, 1) for i, n in enumerate(_PLANES)}
        active = col["active_steps"].clamp_min(1.0)
        grad_score = col["grad_mu"] + col["grad_cov"] + col["grad_amp"]
        return {
            "grad_mu": col["grad_mu"] / active,
            "grad_cov": col["grad_cov"] / active,
            "grad_amp": col["grad_amp"] / active,
            "grad_score": grad_score / active,
            "contrib_score": col["contrib"] / active,
            "active_steps": col["active_steps"].clone(),
        }

    def reset_layer(self, layer_name: str) -> None:
        self._layers[layer_name].zero_()

    def reset_all(self) -> None:
        for name in list(self._layers):
            self.reset_layer(name)
