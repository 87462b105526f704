"""CPU checks of ss_flow's parameter table and random-init weights (the
benchmark's stand-in for a GGUF checkpoint): every linear of the graph is
listed with its shape, and the generated rows are valid GGUF blocks."""
import numpy as np
import pytest

import b2q
import ss_flow


def test_param_specs_cover_the_graph():
    C, nb, T, ch, r = 256, 3, 64, 8, 4
    specs = {name: (kind, shape) for name, kind, shape, _ in ss_flow.param_specs(C, nb, T, ch, r)}
    for e in ("t", "d"):
        assert specs[f"{e}.0"] == ("q", (C, 256)) and specs[f"{e}.2"] == ("q", (C, C))
    assert specs["in.shape"] == ("f", (C, ch)) and specs["pe.shape"] == ("f", (T, C))
    for m, c in ss_flow.POSE:
        assert specs[f"in.{m}"] == ("f", (C, c)) and specs[f"out.{m}"] == ("q", (c, C))
    for i in range(nb):
        assert specs[f"b{i}.adaln"] == ("q", (6 * C, C))
        for g in ss_flow.GROUPS:
            for lin, shp in ss_flow.linear_shapes(C, r * C).items():
                assert specs[f"b{i}.{g}.{lin}"] == ("q", shp)
                assert specs[f"b{i}.{g}.{lin}.b"] == ("f", (shp[0],))
            for v in ("gq", "gk", "n2w", "n2b"):
                assert specs[f"b{i}.{g}.{v}"] == ("f", (C,))
    # every quantized linear is block-quantizable along K
    assert all(shape[1] % 32 == 0 for kind, shape in specs.values() if kind == "q")


@pytest.mark.parametrize("wtype,block", [(b2q.TYPE_Q8_0, 34), (b2q.TYPE_Q4_0, 18)])
def test_random_params_are_valid_gguf_rows(wtype, block):
    import torch
    specs = [("w", "q", (64, 128), (0.0, 0.02)), ("b", "f", (64,), (1.0, 0.1))]
    p = ss_flow.random_params(specs, torch.device("cpu"), wtype, seed=3)
    w = p["w"].numpy()
    assert w.dtype == np.uint8 and w.shape == (64, 128 // 32 * block)
    blocks = w.reshape(64, 4, block)
    d = blocks[:, :, :2].copy().view(np.float16).astype(np.float32)
    assert np.all(np.isfinite(d)) and np.all(d > 0)
    amax = d * (127.0 if wtype == b2q.TYPE_Q8_0 else 8.0)
    assert np.all(amax > 0.02 * 3 * 0.7) and np.all(amax < 0.02 * 3 * 1.3)   # 3 sigma, +-25% jitter
    if wtype == b2q.TYPE_Q8_0:
        assert blocks[:, :, 2:].view(np.int8).min() >= -127
    assert abs(float(p["b"].mean()) - 1.0) < 0.05
