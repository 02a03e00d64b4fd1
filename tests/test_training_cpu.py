"""CPU: the torch restatement of the layer used for training
(burn_gdn2.training.layer_forward), run in float64 with a plain-torch token
loop as its core, against the oracle layer's forward_train (itself pinned to
the reference's golden vectors), to 1e-10.  This pins the graph whose
gradients the GPU training tests compare."""
import numpy as np
import pytest
import torch

import gdn2_oracle as O
from training_ref import torch_loop_core

CFGS = [
    dict(hidden_size=64, num_heads=2, head_dim=32),
    dict(hidden_size=64, num_heads=1, head_dim=32, num_v_heads=2, allow_neg_eigval=True),
    dict(hidden_size=64, num_heads=2, head_dim=16, expand_v=2.0, min_decay=0.9, use_short_conv=False),
]


@pytest.mark.parametrize("cfgd", CFGS)
@pytest.mark.parametrize("gva", ["reference", "grouped"])
def test_layer_forward_matches_oracle(cfgd, gva):
    import burn_gdn2 as bg
    from burn_gdn2 import training

    ocfg = O.Gdn2Config(mode="chunk", **cfgd)
    W = O.init_weights(ocfg, seed=5, dtype=np.float64)
    x = np.random.default_rng(6).standard_normal((2, 19, cfgd["hidden_size"]))
    want = O.Gdn2Layer(ocfg, W, np.float64, gva=gva).forward_train(x)
    cfg = bg.Gdn2Config(mode=bg.Gdn2Mode.Chunk, **cfgd)
    P = {n: torch.tensor(a, dtype=torch.float64) for n, a in W.items()}
    got = training.layer_forward(P, cfg, torch.tensor(x), gva, core=torch_loop_core)
    assert np.abs(got.detach().numpy() - want).max() <= 1e-10 * max(1.0, np.abs(want).max())
