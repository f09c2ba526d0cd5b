"""CPU restatement of the reference autoencoder decoder — TEST INFRASTRUCTURE ONLY.

The oracle the CUDA VAE decoder is checked against.  It restates, in numpy
float32, the reference's CPU decode (iris_vae_decode, iris_vae.c:835-990)
step by step; each function names the reference file:line it follows.  It is
pinned against the reference itself: tests/test_vae_oracle.py decodes the same
latents through the reference compiled from its own sources (oracle/_ref,
ref_vae_decode) and requires the uint8 images to agree.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module.  The product path never does.

Layouts as in the reference: activations NCHW f32 [C, H, W] (batch 1),
convolution weights OIHW, the latent [4 z, h, w] after the 2x2 patchify.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
CH_MULT = (1, 2, 4, 4)   # iris_vae.c:1236
BASE = 128
GROUPS = 32
NUM_RES = 2              # encoder resnets per level; the decoder has NUM_RES + 1


def silu(x):
    """x * sigmoid(x) (swish_inplace -> iris_silu, iris_vae.c:195, iris_kernels.c:610)."""
    return (x / (1.0 + np.exp(-x))).astype(F32)


def group_norm(x, gamma, beta, eps, groups=GROUPS):
    """GroupNorm over [C, H, W] in `groups` channel groups, biased variance
    (iris_group_norm, iris_kernels.c:542-580).  Statistics in float64."""
    c = x.shape[0]
    xg = x.reshape(groups, -1).astype(np.float64)
    mean = xg.mean(1, keepdims=True)
    var = ((xg - mean) ** 2).mean(1, keepdims=True)
    rstd = (1.0 / np.sqrt(var.astype(F32) + F32(eps))).astype(F32)
    y = ((x.reshape(groups, -1) - mean.astype(F32)) * rstd).reshape(x.shape)
    return (y * gamma.reshape(c, 1, 1) + beta.reshape(c, 1, 1)).astype(F32)


def conv2d(x, w, b):
    """Stride-1 convolution, zero padding (k - 1) / 2, OIHW weights
    (vae_conv2d -> iris_conv2d, iris_vae.c:148, iris_kernels.c:363)."""
    cin, hgt, wid = x.shape
    cout, _, kh, kw = w.shape
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    xp = np.pad(x, ((0, 0), (ph, ph), (pw, pw)))
    out = np.zeros((cout, hgt * wid), F32)
    for dy in range(kh):
        for dx in range(kw):
            out += w[:, :, dy, dx] @ xp[:, dy:dy + hgt, dx:dx + wid].reshape(cin, -1)
    if b is not None:
        out += b.reshape(cout, 1)
    return out.reshape(cout, hgt, wid)


def resblock(w, prefix, x, eps):
    """norm1 -> swish -> conv1 -> norm2 -> swish -> conv2, plus the input or
    its 1x1 shortcut conv (resblock_forward, iris_vae.c:203-252)."""
    p = prefix
    if f"{p}.conv_shortcut.weight" in w:
        skip = conv2d(x, w[f"{p}.conv_shortcut.weight"], w[f"{p}.conv_shortcut.bias"])
    else:
        skip = x
    h = silu(group_norm(x, w[f"{p}.norm1.weight"], w[f"{p}.norm1.bias"], eps))
    h = conv2d(h, w[f"{p}.conv1.weight"], w[f"{p}.conv1.bias"])
    h = silu(group_norm(h, w[f"{p}.norm2.weight"], w[f"{p}.norm2.bias"], eps))
    h = conv2d(h, w[f"{p}.conv2.weight"], w[f"{p}.conv2.bias"])
    return (skip + h).astype(F32)


def attnblock(w, prefix, x, eps):
    """Single-head self-attention over the H*W positions, head dim = C, scale
    1/sqrt(C), 1x1-conv projections, residual add (attnblock_forward,
    iris_vae.c:260-354)."""
    p = prefix
    c, hgt, wid = x.shape
    h = group_norm(x, w[f"{p}.group_norm.weight"], w[f"{p}.group_norm.bias"], eps)

    def proj(t, name):
        return conv2d(t, w[f"{p}.{name}.weight"].reshape(c, c, 1, 1), w[f"{p}.{name}.bias"])

    q = proj(h, "to_q").reshape(c, -1).T * F32(1.0 / np.sqrt(c))
    k = proj(h, "to_k").reshape(c, -1).T
    v = proj(h, "to_v").reshape(c, -1).T
    s = q @ k.T
    s = np.exp(s - s.max(1, keepdims=True))
    s = (s / s.sum(1, keepdims=True)).astype(F32)
    o = (s @ v).T.reshape(c, hgt, wid).astype(F32)
    return (x + proj(o, "to_out.0")).astype(F32)


def upsample2x(x):
    """Nearest-neighbour 2x (iris_upsample_nearest, iris_kernels.c:1055)."""
    return np.repeat(np.repeat(x, 2, axis=1), 2, axis=2)


def unpatchify(x, z):
    """[4 z, h, w] -> [z, 2 h, 2 w], channel c * 4 + pi * 2 + pj -> (2 y + pi,
    2 x + pj) (iris_unpatchify, iris_kernels.c:1110-1135)."""
    _, h, wd = x.shape
    return x.reshape(z, 2, 2, h, wd).transpose(0, 3, 1, 4, 2).reshape(z, 2 * h, 2 * wd)


def decode_f32(w, latent, z=32, scaling=0.0, shift=0.0):
    """Latent [4 z, h, w] -> RGB f32 [3, 16 h, 16 w] before the uint8
    conversion (iris_vae_decode, iris_vae.c:835-967).  scaling == 0 selects
    the Flux batch-norm denormalisation with eps 1e-4, else Z-Image's
    x / scaling + shift with eps 1e-6 (iris_vae.c:1245, :855-873)."""
    eps = 1e-6 if scaling != 0.0 else 1e-4
    x = np.asarray(latent, F32)
    if scaling != 0.0:
        x = (x / F32(scaling) + F32(shift)).astype(F32)
    else:
        std = np.sqrt(w["bn.running_var"] + F32(eps)).astype(F32)
        x = (x * std.reshape(-1, 1, 1) + w["bn.running_mean"].reshape(-1, 1, 1)).astype(F32)
    x = unpatchify(x, z)
    if "post_quant_conv.weight" in w:
        x = conv2d(x, w["post_quant_conv.weight"], w["post_quant_conv.bias"])
    x = conv2d(x, w["decoder.conv_in.weight"], w["decoder.conv_in.bias"])
    x = resblock(w, "decoder.mid_block.resnets.0", x, eps)
    x = attnblock(w, "decoder.mid_block.attentions.0", x, eps)
    x = resblock(w, "decoder.mid_block.resnets.1", x, eps)
    for level in range(3, -1, -1):
        up = 3 - level
        for r in range(NUM_RES + 1):
            x = resblock(w, f"decoder.up_blocks.{up}.resnets.{r}", x, eps)
        if level > 0:
            p = f"decoder.up_blocks.{up}.upsamplers.0.conv"
            x = conv2d(upsample2x(x), w[f"{p}.weight"], w[f"{p}.bias"])
    x = silu(group_norm(x, w["decoder.conv_norm_out.weight"], w["decoder.conv_norm_out.bias"], eps))
    return conv2d(x, w["decoder.conv_out.weight"], w["decoder.conv_out.bias"])


def to_rgb8(x):
    """[3, H, W] f32 in [-1, 1] -> uint8 [H, W, 3]: (v + 1) * 0.5 * 255,
    clamped, + 0.5 truncated (iris_vae.c:970-985)."""
    v = ((x.astype(F32) + F32(1.0)) * F32(0.5)) * F32(255.0)
    v = np.clip(v, F32(0.0), F32(255.0))
    return (v + F32(0.5)).astype(np.uint8).transpose(1, 2, 0).copy()


def decode(w, latent, z=32, scaling=0.0, shift=0.0):
    """Latent -> uint8 RGB image [16 h, 16 w, 3] (iris_vae_decode)."""
    return to_rgb8(decode_f32(w, latent, z, scaling, shift))
