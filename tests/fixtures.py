"""Loading helpers for the committed golden fixtures (tests/golden/*.npz)."""
import glob
import json
import os

import numpy as np

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fixture_paths(kind):
    return sorted(glob.glob(os.path.join(GOLDEN, f"{kind}_*.npz")))


def load(path):
    z = dict(np.load(path))
    cfg = json.loads(str(z["cfg"]))
    ad = O.Adapter(int(z["rank"]), float(z["alpha"]), int(z["dora"]), int(z["first_layer"]),
                   int(z["targets"]))
    if str(z["kind"]) == "dit":
        c = O.DitCfg(**{k: cfg[k] for k in ("dim", "layers", "heads", "head_dim", "ff_dim",
                                            "latent_dim", "cond_dim", "time_dim", "n_skip")},
                     norm_eps=cfg["norm_eps"], add_zero_attn=int(cfg["add_zero_attn"]))
    else:
        c = O.LmCfg(**{k: cfg[k] for k in ("dim", "layers", "heads", "head_dim", "ff_dim", "n_q",
                                           "card", "special_token_id", "pos_denominator")},
                    max_period=cfg["max_period"], norm_eps=cfg["norm_eps"])
    return z, c, ad
