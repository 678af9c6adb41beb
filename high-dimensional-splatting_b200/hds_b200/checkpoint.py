"""Checkpoints in the reference's format (gaussian_splatting/main.py:77-94, save_checkpoint).

The reference writes ``torch.save({"params": {name: tensor}, "active_sh_degree", "iteration",
"test_psnr"}, <dir>/model.pt)`` with its GaussianModel's raw parameters: "means" [N,3],
"scales" [N,3] (log-scales), "quats" [N,4] (unnormalised), "opacities" [N,1] (logits), "sh_dc"
[N,1,3] and "sh_rest" [N,15,3] (utils/gaussian.py:47-60).  This module reads such a file into the raw
parameter names the bench and the fused projection use (log_scales, opacity_logits) and writes one
back, so a scene trained by the reference renders here unchanged and the other way round.
"""
from __future__ import annotations

from pathlib import Path

import torch

# reference name -> this package's raw-parameter name
_NAMES = {"means": "means", "scales": "log_scales", "quats": "quats", "opacities": "opacity_logits",
          "sh_dc": "sh_dc", "sh_rest": "sh_rest"}
_SHAPES = {"means": (3,), "scales": (3,), "quats": (4,), "opacities": (1,), "sh_dc": (1, 3)}


def load_checkpoint(path, device="cpu") -> dict:
    """Reads a reference checkpoint (a model.pt file, or the folder holding one).

    Returns {"params": {means, log_scales, quats, opacity_logits, sh_dc, sh_rest} (contiguous float32
    on `device`), "active_sh_degree": int, "iteration": int or None, "test_psnr": float or None}.
    Raises ValueError when a parameter is missing or its shape disagrees with the others."""
    p = Path(path)
    if p.is_dir():
        p = p / "model.pt"
    state = torch.load(p, map_location="cpu", weights_only=True)
    params = state.get("params")
    if not isinstance(params, dict):
        raise ValueError(f"{p}: no 'params' dict (not a reference checkpoint)")
    missing = [k for k in _NAMES if k not in params]
    if missing:
        raise ValueError(f"{p}: missing parameters {missing}")
    n = params["means"].shape[0]
    out = {}
    for ref_name, name in _NAMES.items():
        t = params[ref_name]
        if t.shape[0] != n:
            raise ValueError(f"{p}: {ref_name} has {t.shape[0]} rows, means {n}")
        if ref_name in _SHAPES and tuple(t.shape[1:]) != _SHAPES[ref_name]:
            raise ValueError(f"{p}: {ref_name} has shape {tuple(t.shape)}")
        if ref_name == "sh_rest" and (t.dim() != 3 or t.shape[2] != 3):
            raise ValueError(f"{p}: sh_rest has shape {tuple(t.shape)}")
        out[name] = t.detach().to(device=device, dtype=torch.float32).contiguous()
    return {"params": out, "active_sh_degree": int(state.get("active_sh_degree", 0)),
            "iteration": state.get("iteration"), "test_psnr": state.get("test_psnr")}


def save_checkpoint(path, params: dict, active_sh_degree: int, iteration: int | None = None,
                    test_psnr: float | None = None) -> Path:
    """Writes raw parameters (this package's names) as a reference checkpoint; `path` is the file or
    the folder that receives model.pt.  Returns the file written."""
    p = Path(path)
    if p.suffix != ".pt":
        p.mkdir(parents=True, exist_ok=True)
        p = p / "model.pt"
    inv = {v: k for k, v in _NAMES.items()}
    state = {"params": {inv[k]: v.detach().cpu() for k, v in params.items() if k in inv},
             "active_sh_degree": int(active_sh_degree), "iteration": iteration, "test_psnr": test_psnr}
    torch.save(state, p)
    return p
