"""Loads the golden fixtures of tests/golden/ (made by
tests/golden/make_golden.py from the reference's own CPU build)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN, name)) as f:
        return {k: f[k] for k in f.files}


def _scalar(v):
    v = np.asarray(v)
    return v.item() if v.ndim == 0 else v


def moe_layer():
    """(layer dict in make_moe_layer's form, hidden, out, ids, contributions)."""
    f = load("moe_layer.npz")
    layer = {k[4:]: _scalar(v) for k, v in f.items() if k.startswith("dim_")}
    for k, v in f.items():
        if not k.startswith("dim_") and k not in ("hidden", "out", "ids", "contributions"):
            layer[k] = v
    for k in ("hidden", "inter", "experts", "top_k", "shared_inter", "activation"):
        layer[k] = int(layer[k])
    for k in ("situ_beta", "situ_linear_beta"):
        layer[k] = float(layer[k])
    return layer, f["hidden"], f["out"], f["ids"], f["contributions"]


def latent_moe():
    """(layer dict with latent fields, fixture dict)."""
    f = load("latent_moe.npz")
    skip = ("prefix", "block", "residual_norm", "residual_proj", "post_norm", "eps", "out", "ids", "contributions")
    layer = {k[4:]: _scalar(v) for k, v in f.items() if k.startswith("dim_")}
    for k, v in f.items():
        if not k.startswith("dim_") and k not in skip:
            layer[k] = v
    for k in ("hidden", "inter", "experts", "top_k", "shared_inter", "activation", "latent"):
        layer[k] = int(layer[k])
    for k in ("situ_beta", "situ_linear_beta", "latent_eps"):
        layer[k] = float(layer[k])
    return layer, f


def official_layer():
    """(layer dict in make_layer's form with a LatentMoE, fixture dict)."""
    f = load("official_layer.npz")
    layer = {k[5:]: f[k] for k in f if k.startswith("norm_")}
    layer["rms_eps"] = float(f["rms_eps"])
    kda = {k[4:]: _scalar(f[k]) for k in f if k.startswith("kda_")}
    moe = {k[4:]: _scalar(f[k]) for k in f if k.startswith("moe_")}
    for k in ("hidden", "heads", "head_dim", "conv_width"):
        kda[k] = int(kda[k])
    for k in ("eps", "gate_lower_bound"):
        kda[k] = float(kda[k])
    for k in ("hidden", "inter", "experts", "top_k", "shared_inter", "activation", "latent"):
        moe[k] = int(moe[k])
    for k in ("situ_beta", "situ_linear_beta", "latent_eps"):
        moe[k] = float(moe[k])
    layer["kda"], layer["moe"] = kda, moe
    layer["hidden"] = kda["hidden"]
    return layer, f


def kda_block():
    """(weights dict in make_kda_weights's form, fixture dict)."""
    f = load("kda_block.npz")
    w = {k[2:]: v for k, v in f.items() if k.startswith("w_")}
    for k, v in f.items():
        if k.startswith("dim_"):
            w[k[4:]] = _scalar(v)
    for k in ("hidden", "heads", "head_dim", "conv_width"):
        w[k] = int(w[k])
    for k in ("eps", "gate_lower_bound"):
        w[k] = float(w[k])
    return w, f
