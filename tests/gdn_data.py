"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (2 and 4).  numpy RandomState
keeps them identical on every machine.

Distributions: mixed_qkv (the in_proj_qkv output) and z ~ N(0,1);
g = -softplus(N(0,1)); beta = sigmoid(N(0,1)); S0 ~ N(0, 0.02^2); conv weight
~ N(0, 0.5^2) (unspecified by the configs; this scale keeps conv outputs O(1));
norm weight 1 + N(0, 0.1^2) (init is ones); conv state 0.5*N(0,1).
"""
import numpy as np


def softplus(x):
    return np.log1p(np.exp(x))


def gdn_inputs(seed, B, Hk, Hv, steps, K=4, D=128):
    rng = np.random.RandomState(seed)
    C = 2 * Hk * D + Hv * D
    f = np.float32
    return dict(
        x=rng.randn(steps, B, C).astype(f),
        z=rng.randn(steps, B, Hv * D).astype(f),
        g=(-softplus(rng.randn(steps, B, Hv))).astype(f),
        beta=(1.0 / (1.0 + np.exp(-rng.randn(steps, B, Hv)))).astype(f),
        S0=(0.02 * rng.randn(B, Hv, D, D)).astype(f),
        conv_w=(0.5 * rng.randn(C, K)).astype(f),
        norm_w=(1.0 + 0.1 * rng.randn(D)).astype(f),
        conv0=(0.5 * rng.randn(B, C, K - 1)).astype(f),
    )


def gqa_inputs(seed, B, Hq, Hkv, steps, L0, cap, D=256, wscale=0.0):
    """K/V cache ~ N(0,1) for the first L0 tokens; per step q_gate, k, v ~ N(0,1);
    q_norm/k_norm weights 0 (init) or N(0, wscale^2)."""
    rng = np.random.RandomState(seed)
    f = np.float32
    Kc = np.zeros((B, Hkv, cap, D), f)
    Vc = np.zeros((B, Hkv, cap, D), f)
    Kc[:, :, :L0] = rng.randn(B, Hkv, L0, D)
    Vc[:, :, :L0] = rng.randn(B, Hkv, L0, D)
    return dict(
        K=Kc, V=Vc,
        qg=rng.randn(steps, B, Hq, 2 * D).astype(f),
        kn=rng.randn(steps, B, Hkv, D).astype(f),
        vn=rng.randn(steps, B, Hkv, D).astype(f),
        qn_w=(wscale * rng.randn(D)).astype(f),
        kn_w=(wscale * rng.randn(D)).astype(f),
    )
