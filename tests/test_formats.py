"""On-disk formats: a checkpoint written by the reference's
GaussianModel.save_checkpoint loads, a checkpoint written here has the
reference's key set, and file names parse to the reference's dictionaries."""
import json
import os

import torch

from cuda_rasterizer import formats as FM

HERE = os.path.join(os.path.dirname(__file__), "golden")


def test_reference_checkpoint_loads_and_round_trips(tmp_path):
    ck = FM.load_checkpoint(os.path.join(HERE, "formats_checkpoint.pt"))
    assert ck["iteration"] == 1234 and ck["sh_degree"] == 3 and ck["active_sh_degree"] == 2
    assert ck["means"].shape == (50, 3) and ck["opacities"].shape == (50, 1)
    assert ck["sh_coeffs"].shape == (50, 16) and ck["optimizer_state"] is None
    path = str(tmp_path / "ck.pt")
    FM.save_checkpoint(path, ck["means"], ck["scales"], ck["rotations"], ck["opacities"], ck["sh_coeffs"],
                       iteration=7, sh_degree=3, active_sh_degree=2, optimizer_state={"lr": 1e-3})
    raw = torch.load(path, weights_only=False)
    ref = torch.load(os.path.join(HERE, "formats_checkpoint.pt"), weights_only=False)
    assert set(raw) == set(ref) | {"optimizer_state"}
    back = FM.load_checkpoint(path)
    for k in ("means", "scales", "rotations", "opacities", "sh_coeffs"):
        assert torch.equal(back[k], ck[k])
    assert back["iteration"] == 7 and back["optimizer_state"] == {"lr": 1e-3}


def test_file_names_parse_like_the_reference():
    with open(os.path.join(HERE, "formats_names.json")) as fh:
        ref = json.load(fh)
    for name, expected in ref.items():
        assert FM.parse_sar_filename(name) == expected, name
    v = FM.view_from_filename("inc_30.0-track_45.5-height_5000-squint_0.0-rr_0.3-ar_0.3.png", 128, 96)
    assert v == (0.0, 0.0, 5000.0, 45.5, 30.0, 0.0, 0.3, 0.3, 128, 96)
