"""ctypes loader for the reference compiled from its own sources — TEST INFRASTRUCTURE ONLY.

oracle/Makefile builds oracle/_ref/libiris_ref_{generic,blas}.so from the
unmodified reference C files plus oracle/ref_harness.c.  This module binds
the harness entry points (see ref_harness.c for the reference function each
one calls).  Used to generate golden fixtures, to pin the numpy oracle and as
bench.py's reference (CPU) arm.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_fp = C.POINTER(C.c_float)


def _f(a):
    return a.ctypes.data_as(_fp)


class RefLib:
    def __init__(self, variant: str = "blas"):
        path = os.path.join(REF_DIR, f"libiris_ref_{variant}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle` where the reference tree exists")
        self.lib = L = C.CDLL(path)
        L.ref_flux_load.restype = C.c_void_p
        L.ref_flux_load.argtypes = [C.c_char_p]
        L.ref_flux_load_mmap.restype = C.c_void_p
        L.ref_flux_load_mmap.argtypes = [C.c_char_p]
        L.ref_flux_free.argtypes = [C.c_void_p]
        L.ref_flux_config.argtypes = [C.c_void_p, _fp]
        L.ref_flux_forward.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int, C.c_float, _fp]
        L.ref_flux_forward_refs.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int,
                                            C.c_int, C.c_int, _fp, C.c_int, C.c_float, _fp]
        L.ref_flux_temb.argtypes = [C.c_void_p, C.c_float, _fp]
        L.ref_flux_mods.argtypes = [C.c_void_p, _fp, _fp, _fp, _fp, _fp]
        L.ref_flux_rope_img.argtypes = [C.c_void_p, C.c_int, C.c_int, _fp, _fp]
        L.ref_flux_rope_txt.argtypes = [C.c_void_p, C.c_int, _fp, _fp]
        L.ref_flux_double_block.argtypes = [C.c_void_p, C.c_int, _fp, _fp, _fp, _fp,
                                            C.c_int, C.c_int, C.c_int]
        L.ref_flux_single_block.argtypes = [C.c_void_p, C.c_int, _fp, _fp, C.c_int, C.c_int, C.c_int]
        L.ref_init_noise.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int64, _fp]
        L.ref_official_schedule.argtypes = [C.c_int, C.c_int, _fp]
        L.ref_zimage_schedule.argtypes = [C.c_int, C.c_int, _fp]
        L.ref_sample_euler.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, _fp, C.c_int,
                                       _fp, C.c_int, _fp]
        L.ref_sample_euler_cfg.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, _fp, C.c_int,
                                           _fp, C.c_int, C.c_float, _fp, C.c_int, _fp]
        L.ref_zi_load.restype = C.c_void_p
        L.ref_zi_load.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.c_float]
        L.ref_zi_free.argtypes = [C.c_void_p]
        L.ref_zi_forward.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_float, _fp, C.c_int,
                                     C.c_int, _fp]
        L.ref_sample_euler_zimage.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                              _fp, C.c_int, _fp, C.c_int, _fp]
        L.ref_set_threads.argtypes = [C.c_int]
        L.ref_qwen3_forward.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int, _fp,
                                        C.c_int]
        L.ref_qwen3_last_forward_s.restype = C.c_double
        L.ref_vae_decode.argtypes = [C.c_char_p, C.c_int, _fp, C.c_int, C.c_int, C.POINTER(C.c_uint8),
                                     C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ref_vae_decode_ex.argtypes = [C.c_char_p, C.c_int, C.c_float, C.c_float, _fp, C.c_int, C.c_int,
                                        C.POINTER(C.c_uint8), C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ref_ip_perceive.argtypes = [C.c_char_p, _fp, C.c_int, _fp, C.c_int]
        L.ref_ip_get_kv.argtypes = [C.c_char_p, C.c_int, _fp, _fp, _fp]
        L.ref_ip_inject.argtypes = [C.c_char_p, C.c_int, _fp, C.c_int, _fp, _fp, _fp, C.c_char_p, C.c_int,
                                    C.c_int]
        L.ref_flux_set_ip.argtypes = [C.c_void_p, C.c_char_p, _fp, C.c_int, C.c_float]
        L.ref_flux_set_ip_schedule.argtypes = [C.c_void_p, C.c_char_p]
        L.ref_flux_clear_ip.argtypes = [C.c_void_p]
        L.ref_flux_set_sref_csd.argtypes = [C.c_void_p, C.c_char_p, _fp, C.c_int, C.c_float]
        L.ref_flux_set_sref_bands.argtypes = [C.c_void_p, C.c_float, C.c_float]
        L.ref_flux_set_lora.argtypes = [C.c_void_p, C.c_char_p, C.c_float]
        L.ref_flux_clear_lora.argtypes = [C.c_void_p]
        L.ref_lora_get.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.POINTER(C.c_int), _fp, C.c_size_t, _fp, C.c_size_t]

    def ip_perceive(self, bundle: str, feats: np.ndarray, tokens: int, hidden: int) -> np.ndarray:
        f = np.ascontiguousarray(feats, np.float32)
        out = np.zeros(tokens * hidden, np.float32)
        n = f.shape[0] if f.ndim > 1 else 1
        rc = self.lib.ref_ip_perceive(bundle.encode(), _f(f), n, _f(out), out.size)
        if rc < 0:
            raise RuntimeError(f"reference perceive failed ({rc})")
        return out.reshape(tokens, hidden)

    def ip_get_kv(self, bundle: str, blk: int, embeds: np.ndarray):
        e = np.ascontiguousarray(embeds, np.float32)
        k, v = np.zeros_like(e), np.zeros_like(e)
        if self.lib.ref_ip_get_kv(bundle.encode(), blk, _f(e), _f(k), _f(v)):
            raise RuntimeError("reference get_kv failed")
        return k, v

    def ip_inject(self, bundle: str, blk: int, q, k, v, hidden, sched=None, step=0, nsteps=0):
        q, k, v = (np.ascontiguousarray(x, np.float32) for x in (q, k, v))
        h = np.ascontiguousarray(hidden, np.float32).copy()
        rc = self.lib.ref_ip_inject(bundle.encode(), blk, _f(q), q.shape[0], _f(k), _f(v), _f(h),
                                    sched.encode() if sched else None, step, nsteps)
        if rc:
            raise RuntimeError(f"reference inject failed ({rc})")
        return h

    def lora_get(self, path: str, n_double: int, n_single: int, hidden: int, kind: int, block: int,
                 cap: int = 1 << 22):
        """(A, B) of one adapter of the reference's lora_load table, None if absent,
        raises if lora_load failed."""
        dims = (C.c_int * 3)()
        a = np.zeros(cap, np.float32)
        b = np.zeros(cap, np.float32)
        rc = self.lib.ref_lora_get(path.encode(), n_double, n_single, hidden, kind, block, dims,
                                   _f(a), cap, _f(b), cap)
        if rc < 0:
            raise RuntimeError(f"reference lora_load failed on {path}")
        if rc == 0:
            return None
        r, i, o = dims
        return a[:r * i].reshape(r, i).copy(), b[:o * r].reshape(o, r).copy()

    def qwen3_forward(self, model_dir: str, ids, mask, text_dim: int, zimage: bool = False) -> np.ndarray:
        """Reference CPU text encoder (qwen3_model_load + qwen3_forward) -> [seq, text_dim]."""
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ascontiguousarray(mask, np.int32)
        seq = len(ids)
        out = np.zeros(seq * text_dim, np.float32)
        ip = C.POINTER(C.c_int)
        rc = self.lib.ref_qwen3_forward(model_dir.encode(), int(zimage), ids.ctypes.data_as(ip),
                                        mask.ctypes.data_as(ip), seq, _f(out), seq * text_dim)
        if rc != text_dim:
            raise RuntimeError(f"reference qwen3_forward failed ({rc})")
        self.qwen3_forward_s = self.lib.ref_qwen3_last_forward_s()
        return out.reshape(seq, text_dim)

    def set_threads(self, n: int):
        self.lib.ref_set_threads(n)

    def vae_decode(self, vae_file: str, latent: np.ndarray, z: int = 32, scaling: float = 0.0,
                   shift: float = 0.0) -> np.ndarray:
        """Reference CPU decode (iris_vae_decode) of a [4z, h, w] latent -> uint8 [16h, 16w, 3].
        scaling != 0: Z-Image latent scaling/shift instead of batch-norm statistics."""
        lat = np.ascontiguousarray(latent, np.float32)
        _, h, w = lat.shape
        out = np.zeros(3 * 16 * h * 16 * w, np.uint8)
        ow, oh = C.c_int(0), C.c_int(0)
        rc = self.lib.ref_vae_decode_ex(vae_file.encode(), z, scaling, shift, _f(lat), h, w,
                                        out.ctypes.data_as(C.POINTER(C.c_uint8)), C.byref(ow), C.byref(oh))
        if rc != 3:
            raise RuntimeError(f"reference VAE decode failed ({rc})")
        return out[: oh.value * ow.value * 3].reshape(oh.value, ow.value, 3)


def psnr(a: np.ndarray, b: np.ndarray) -> float:
    """PSNR (dB) of two uint8 images."""
    mse = np.mean((a.astype(np.float64) - b.astype(np.float64)) ** 2)
    return float("inf") if mse == 0 else float(10.0 * np.log10(255.0 ** 2 / mse))


class RefFlux:
    """A reference Flux transformer loaded from a model directory."""

    def __init__(self, ref: RefLib, model_dir: str, mmap: bool = False):
        self.ref = ref
        load = ref.lib.ref_flux_load_mmap if mmap else ref.lib.ref_flux_load
        self.h = load(model_dir.encode())
        if not self.h:
            raise RuntimeError(f"reference failed to load {model_dir}")
        cfg = np.zeros(10, np.float32)
        ref.lib.ref_flux_config(self.h, _f(cfg))
        (self.hidden, self.heads, self.head_dim, self.mlp, self.n_double, self.n_single,
         self.text_dim, self.channels) = (int(x) for x in cfg[:8])
        self.theta = float(cfg[8])

    def close(self):
        if self.h:
            self.ref.lib.ref_flux_free(self.h)
            self.h = None

    def forward(self, latent, txt, t):
        c, h, w = latent.shape
        lat = np.ascontiguousarray(latent, np.float32)
        tx = np.ascontiguousarray(txt, np.float32)
        out = np.zeros_like(lat)
        rc = self.ref.lib.ref_flux_forward(self.h, _f(lat), h, w, _f(tx), tx.shape[0], t, _f(out))
        assert rc == 0
        return out

    def set_ip(self, bundle: str, feats: np.ndarray, scale_mult: float = 1.0) -> int:
        f = np.ascontiguousarray(feats, np.float32)
        return self.ref.lib.ref_flux_set_ip(self.h, bundle.encode(), _f(f), f.shape[0] if f.ndim > 1 else 1,
                                            scale_mult)

    def set_ip_schedule(self, spec: str) -> int:
        return self.ref.lib.ref_flux_set_ip_schedule(self.h, spec.encode())

    def clear_ip(self):
        self.ref.lib.ref_flux_clear_ip(self.h)

    def set_sref_csd(self, csdmod, csd, scale) -> int:
        c = np.ascontiguousarray(csd, np.float32).ravel()
        return self.ref.lib.ref_flux_set_sref_csd(self.h, csdmod.encode() if csdmod else None, _f(c), c.size, scale)

    def set_sref_bands(self, shf, slf):
        self.ref.lib.ref_flux_set_sref_bands(self.h, shf, slf)

    def set_lora(self, path: str, scale: float) -> bool:
        return self.ref.lib.ref_flux_set_lora(self.h, path.encode(), scale) == 0

    def clear_lora(self):
        self.ref.lib.ref_flux_clear_lora(self.h)

    def forward_refs(self, latent, refs, txt, t):
        c, h, w = latent.shape
        lat = np.ascontiguousarray(latent, np.float32)
        rl = np.ascontiguousarray(np.stack(refs), np.float32)
        tx = np.ascontiguousarray(txt, np.float32)
        out = np.zeros_like(lat)
        rc = self.ref.lib.ref_flux_forward_refs(self.h, _f(lat), h, w, _f(rl), len(refs),
                                                refs[0].shape[1], refs[0].shape[2],
                                                _f(tx), tx.shape[0], t, _f(out))
        assert rc == 0
        return out

    def temb(self, t):
        out = np.zeros(self.hidden, np.float32)
        self.ref.lib.ref_flux_temb(self.h, t, _f(out))
        return out

    def mods(self, t_emb):
        H = self.hidden
        a, b, c, d = (np.zeros(n * H, np.float32) for n in (6, 6, 3, 2))
        self.ref.lib.ref_flux_mods(self.h, _f(np.ascontiguousarray(t_emb, np.float32)),
                                   _f(a), _f(b), _f(c), _f(d))
        return dict(dbl_img=a, dbl_txt=b, single=c, final=d)

    def double_block(self, i, img, txt, mod_img, mod_txt, ph, pw):
        img = np.ascontiguousarray(img, np.float32).copy()
        txt = np.ascontiguousarray(txt, np.float32).copy()
        rc = self.ref.lib.ref_flux_double_block(self.h, i, _f(img), _f(txt),
                                                _f(np.ascontiguousarray(mod_img, np.float32)),
                                                _f(np.ascontiguousarray(mod_txt, np.float32)),
                                                ph, pw, txt.shape[0])
        assert rc == 0
        return img, txt

    def single_block(self, i, hidden, t_emb, ph, pw, txt_seq):
        hid = np.ascontiguousarray(hidden, np.float32).copy()
        rc = self.ref.lib.ref_flux_single_block(self.h, i, _f(hid),
                                                _f(np.ascontiguousarray(t_emb, np.float32)),
                                                ph, pw, txt_seq)
        assert rc == 0
        return hid

    def sample_euler(self, z, txt, schedule):
        c, h, w = z.shape
        zz = np.ascontiguousarray(z, np.float32).copy()
        tx = np.ascontiguousarray(txt, np.float32)
        sc = np.ascontiguousarray(schedule, np.float32)
        out = np.zeros_like(zz)
        rc = self.ref.lib.ref_sample_euler(self.h, _f(zz), c, h, w, _f(tx), tx.shape[0], _f(sc),
                                           len(sc) - 1, _f(out))
        assert rc == 0
        return out

    def sample_euler_cfg(self, z, txt_c, txt_u, g, schedule):
        c, h, w = z.shape
        zz = np.ascontiguousarray(z, np.float32).copy()
        tc = np.ascontiguousarray(txt_c, np.float32)
        tu = np.ascontiguousarray(txt_u, np.float32)
        sc = np.ascontiguousarray(schedule, np.float32)
        out = np.zeros_like(zz)
        rc = self.ref.lib.ref_sample_euler_cfg(self.h, _f(zz), c, h, w, _f(tc), tc.shape[0],
                                               _f(tu), tu.shape[0], g, _f(sc), len(sc) - 1, _f(out))
        assert rc == 0
        return out


def ref_init_noise(ref: RefLib, c, h, w, seed):
    out = np.zeros((c, h, w), np.float32)
    assert ref.lib.ref_init_noise(c, h, w, seed, _f(out)) == 0
    return out


def ref_official_schedule(ref: RefLib, steps, seq):
    out = np.zeros(steps + 1, np.float32)
    assert ref.lib.ref_official_schedule(steps, seq, _f(out)) == 0
    return out


def ref_zimage_schedule(ref: RefLib, steps, seq):
    out = np.zeros(steps + 1, np.float32)
    assert ref.lib.ref_zimage_schedule(steps, seq, _f(out)) == 0
    return out


class RefZImage:
    """A reference Z-Image transformer loaded from a model directory."""

    def __init__(self, ref: RefLib, model_dir: str, cfg: dict):
        self.ref = ref
        self.cfg = cfg
        arr = (C.c_int * 10)(cfg["dim"], cfg["dim"] // 128, cfg["n_layers"], cfg["n_refiner"],
                             cfg["cap_feat_dim"], cfg["in_channels"], cfg["patch_size"], *cfg["axes_dims"])
        self.h = ref.lib.ref_zi_load(model_dir.encode(), arr, float(cfg["rope_theta"]))
        if not self.h:
            raise RuntimeError(f"reference failed to load {model_dir}")

    def close(self):
        if self.h:
            self.ref.lib.ref_zi_free(self.h)
            self.h = None

    def forward(self, latent, cap, t):
        c, h, w = latent.shape
        lat = np.ascontiguousarray(latent, np.float32)
        cp = np.ascontiguousarray(cap, np.float32)
        out = np.zeros_like(lat)
        rc = self.ref.lib.ref_zi_forward(self.h, _f(lat), h, w, t, _f(cp), cp.shape[0], c, _f(out))
        assert rc == 0
        return out

    def sample_euler(self, z, cap, schedule):
        c, h, w = z.shape
        zz = np.ascontiguousarray(z, np.float32).copy()
        cp = np.ascontiguousarray(cap, np.float32)
        sc = np.ascontiguousarray(schedule, np.float32)
        out = np.zeros_like(zz)
        rc = self.ref.lib.ref_sample_euler_zimage(self.h, _f(zz), c, h, w, self.cfg["patch_size"], _f(cp),
                                                  cp.shape[0], _f(sc), len(sc) - 1, _f(out))
        assert rc == 0
        return out
