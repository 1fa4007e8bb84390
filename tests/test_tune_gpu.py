"""GPU: the per-shape variant table (scx_tune.py, the counterpart of the reference's
spectral_conv_combo/tune.py).  Every variant the library offers for a shape gives the default's
result, the tuner returns entries for the shape, and a saved table reloads and is applied."""

from __future__ import annotations

import pytest
import torch

import _scx
import scx_data
import scx_tune
import spectral_conv_ops

pytestmark = pytest.mark.gpu


def _forward(x, w1, w2, c, device):
    return spectral_conv_ops.spectral_conv2d(x.to(device), w1.to(device), w2.to(device), c["m1"], c["m2"])


@pytest.mark.parametrize("name", ["spectral_b20_c32_64x64_m12", "spectral_b16_c64_256x256_m32"])
def test_every_variant_matches_the_default(name, cuda_device):
    lib = _scx.lib
    x, w1, w2, c = scx_data.make_spectral_case(name, batch=4)
    H, W, m1, m2 = c["H"], c["W"], c["m1"], c["m2"]
    lib.scx_clear_variants()
    ref = _forward(x, w1, w2, c, cuda_device)
    scale = ref.abs().max().item()
    mask = lib.scx_dft_variants(H, W, m1, m2)
    try:
        for code in (1, 2, 3):
            if mask & (1 << code):
                assert lib.scx_set_dft_variant(H, W, m1, m2, code) == 0
                got = _forward(x, w1, w2, c, cuda_device)
                assert (got - ref).abs().max().item() <= 1e-5 * scale, code
        lib.scx_set_dft_variant(H, W, m1, m2, 0)
        for v in list(range(scx_tune.MIX_RING_SHAPES + 1)) + [scx_tune.MIX_TC]:
            assert lib.scx_set_mix_variant(2, c["B"], c["Cin"], c["Cout"], m1 * m2, v) == 0
            got = _forward(x, w1, w2, c, cuda_device)
            assert (got - ref).abs().max().item() <= 1e-5 * scale, v
    finally:
        lib.scx_clear_variants()


def test_tuner_writes_a_table_that_reloads(cuda_device, tmp_path):
    lib = _scx.lib
    x, w1, w2, c = scx_data.make_spectral_case("spectral_b20_c32_64x64_m12")
    try:
        d, m, times = scx_tune.tune_spectral(x, w1, w2, c, cuda_device, reps=3)
        assert d["variant"] in ("auto", "ffma", "tensor", "folded") and "default" in times
        table = scx_tune.empty_table()
        scx_tune.merge(table, d, "dft")
        scx_tune.merge(table, m, "mix")
        path = scx_tune.save(table, tmp_path / "t.json")
        lib.scx_clear_variants()
        scx_tune.load(path)
        assert lib.scx_get_variant(1, 2, c["B"], c["Cin"], c["Cout"], c["m1"] * c["m2"]) == m["variant"]
        ref = _forward(x, w1, w2, c, cuda_device)  # runs with the tuned variants
        assert torch.isfinite(ref).all()
    finally:
        lib.scx_clear_variants()
