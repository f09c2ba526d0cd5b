"""Golden-fixture case table and seeded inputs, shared by make_golden.py and
the tests.  Inputs are regenerated from their seeds instead of being stored;
the .npz files hold the reference's outputs (and the reference RNG's noise).
"""
from __future__ import annotations

import numpy as np

FLUX_CASES = {
    # tiny: 2 heads, 1 double + 2 single blocks; unit QK-norm scales exercise softmax
    "flux_tiny": dict(cfg=dict(num_attention_heads=2, attention_head_dim=128, num_layers=1,
                               num_single_layers=2, joint_attention_dim=64, in_channels=128,
                               mlp_ratio=3.0, rope_theta=2000.0),
                      seed=7, std=0.05, norm_mode="unit", img=(4, 4), txt=8),
    # BASELINE-style init: every tensor N(0, 0.02), norm scales included
    "flux_tiny_n002": dict(cfg=dict(num_attention_heads=2, attention_head_dim=128, num_layers=1,
                                    num_single_layers=1, joint_attention_dim=64, in_channels=128,
                                    mlp_ratio=3.0, rope_theta=2000.0),
                           seed=11, std=0.02, norm_mode="random", img=(4, 4), txt=8),
    # small: ragged token counts (not multiples of 128), 2 + 2 blocks
    "flux_small": dict(cfg=dict(num_attention_heads=4, attention_head_dim=128, num_layers=2,
                                num_single_layers=2, joint_attention_dim=128, in_channels=128,
                                mlp_ratio=3.0, rope_theta=2000.0),
                       seed=3, std=0.04, norm_mode="unit", img=(6, 10), txt=37),
}


def rng_inputs(seed, c, h, w, txt, text_dim):
    r = np.random.default_rng(seed)
    lat = r.standard_normal((c, h, w)).astype(np.float32)
    ctx = r.standard_normal((txt, text_dim)).astype(np.float32)
    return lat, ctx




def block_inputs(spec, hidden):
    """Seeded hidden states fed to one double and one single block."""
    h, w = spec["img"]
    r = np.random.default_rng(spec["seed"] + 200)
    img_h = r.standard_normal((h * w, hidden)).astype(np.float32)
    txt_h = r.standard_normal((spec["txt"], hidden)).astype(np.float32)
    return img_h, txt_h


def ref_inputs(channels, txt_shape):
    """Two reference latents [C, 2, 3] and an unconditional context."""
    rr = np.random.default_rng(5)
    refs = [rr.standard_normal((channels, 2, 3)).astype(np.float32) for _ in range(2)]
    ctx_u = rr.standard_normal(txt_shape).astype(np.float32)
    return refs, ctx_u


ZIMAGE_CASES = {
    # tiny: dim 256 (2 heads), 1 refiner each, 1 main layer; 30 image tokens (pad 2), 7 caption tokens (pad 25)
    "zimage_tiny": dict(cfg=dict(dim=256, n_heads=2, n_layers=1, n_refiner=1, cap_feat_dim=64, in_channels=16,
                                 patch_size=2, rope_theta=256.0, axes_dims=[32, 48, 48], ffn_dim=768,
                                 adaln_dim=256, t_mid=256),
                        seed=3, std=0.05, norm_mode="unit", latent=(16, 10, 12), cap=7),
    # small: dim 512, 2 refiners each, 2 main layers; 64 image tokens (no pad), 40 caption tokens (pad 24)
    "zimage_small": dict(cfg=dict(dim=512, n_heads=4, n_layers=2, n_refiner=2, cap_feat_dim=128, in_channels=16,
                                  patch_size=2, rope_theta=256.0, axes_dims=[32, 48, 48], ffn_dim=1536,
                                  adaln_dim=256, t_mid=512),
                         seed=9, std=0.04, norm_mode="unit", latent=(16, 16, 16), cap=40),
}


def zimage_inputs(spec):
    r = np.random.default_rng(spec["seed"] + 100)
    lat = r.standard_normal(spec["latent"]).astype(np.float32)
    cap = r.standard_normal((spec["cap"], spec["cfg"]["cap_feat_dim"])).astype(np.float32)
    return lat, cap
