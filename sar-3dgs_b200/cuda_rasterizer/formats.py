"""On-disk formats of SAR-3DGS used around the rasterizer: the Gaussian-model
checkpoint dictionary (GaussianModel.save_checkpoint / load_checkpoint,
gaussian_model.py:353-408) and the SAR image file-name convention that
carries the radar parameters of a view (parse_sar_filename,
scene/dataset_readers.py:52-96). Checkpoints written by either side load in
the other; file names parse to the same dictionaries, and view_from_filename
turns one into the rasterizer's view tuple.
"""
import re
from typing import Dict, Optional, Tuple

import torch

__all__ = ["save_checkpoint", "load_checkpoint", "parse_sar_filename", "view_from_filename"]

# The key set of the reference's checkpoint dictionary.
_TENSORS = ("means", "scales", "rotations", "opacities", "sh_coeffs")


def save_checkpoint(file_path: str, means, scales, rotations, opacities, sh_coeffs, iteration: int = 0,
                    sh_degree: int = 3, active_sh_degree: int = 0, optimizer_state: dict = None) -> None:
    """Writes the reference's checkpoint dictionary (tensors on the CPU)."""
    ck = {"iteration": iteration}
    for k, t in zip(_TENSORS, (means, scales, rotations, opacities, sh_coeffs)):
        ck[k] = t.detach().cpu()
    ck.update({"sh_degree": sh_degree, "active_sh_degree": active_sh_degree,
               "num_gaussians": int(means.shape[0])})
    if optimizer_state is not None:
        ck["optimizer_state"] = optimizer_state
    torch.save(ck, file_path)


def load_checkpoint(file_path: str, device=None) -> Dict:
    """Reads a checkpoint dictionary: the five parameter tensors on `device`,
    sh_degree and active_sh_degree (defaults 3 and 0 as the reference reads
    them), iteration and optimizer_state (or None)."""
    device = torch.device("cpu") if device is None else torch.device(device)
    ck = torch.load(file_path, map_location="cpu", weights_only=False)
    out = {k: ck[k].to(device) for k in _TENSORS}
    out["sh_degree"] = ck.get("sh_degree", 3)
    out["active_sh_degree"] = ck.get("active_sh_degree", 0)
    out["iteration"] = ck.get("iteration", 0)
    out["optimizer_state"] = ck.get("optimizer_state", None)
    return out


_NEW = re.compile(r"inc_([n\d.]+)-track_([n\d.]+)-height_(\d+)-squint_([n\d.]+)-rr_([\d.]+)-ar_([\d.]+)\.png")
_OLD = re.compile(r"elev-([\d.]+)-azim-(-?[\d.]+)-A\.png")


def _signed(val: str) -> float:
    return -float(val[1:]) if val.startswith("n") else float(val)


def parse_sar_filename(filename: str) -> Optional[Dict]:
    """Radar parameters from a file name: 'inc_{inc}-track_{track}-height_{h}-
    squint_{squint}-rr_{rr}-ar_{ar}.png' (an 'n' prefix marks a negative
    value) or the older 'elev-{inc}-azim-{track}-A.png' (height 10 km, squint
    0, 0.3 m resolutions); None otherwise."""
    m = _NEW.match(filename)
    if m:
        return {"incidence": float(m.group(1)), "track": _signed(m.group(2)), "height": float(m.group(3)),
                "squint": _signed(m.group(4)), "range_resolution": float(m.group(5)),
                "azimuth_resolution": float(m.group(6)), "format": "new"}
    m = _OLD.match(filename)
    if m:
        return {"incidence": float(m.group(1)), "track": float(m.group(2)), "height": 10000.0,
                "squint": 0.0, "range_resolution": 0.3, "azimuth_resolution": 0.3, "format": "old"}
    return None


def view_from_filename(filename: str, range_samples: int, azimuth_samples: int) -> Optional[Tuple]:
    """(radar_x, radar_y, radar_z, track, incidence, squint, rho_r, rho_a, Nr,
    Na) for render_sar / SARRasterizer; the library derives the radar
    position from the altitude and the angles."""
    p = parse_sar_filename(filename)
    if p is None:
        return None
    return (0.0, 0.0, p["height"], p["track"], p["incidence"], p["squint"], p["range_resolution"],
            p["azimuth_resolution"], int(range_samples), int(azimuth_samples))
