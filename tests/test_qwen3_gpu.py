"""Qwen3 text encoder on the GPU through the C ABI (iris_cuda_qwen3_*) against
the numpy oracle (pinned to the reference encoder by tests/test_qwen3_oracle.py)
and the reference's own CPU encoder (oracle/_ref).

Gate: rel-L2 <= 1e-2 (north_star's bf16 tolerance) over the real tokens'
rows of every extracted hidden state, <= 1.5e-2 over all rows.  The padded
rows (the reference keeps them; they feed the transformer) drift further: a
numpy restatement that only rounds to bf16 where this encoder does (GEMM
operands, Q/K/V, P, attention and MLP outputs) already lands at 1.05e-2 after
27 layers on the 512-token, 77-real-token prompt (1.02e-2 on padded rows,
0.54-0.70 % on real ones), and the GPU matches that figure.  Covers causal
grouped-query attention (4 query heads on 2 key/value heads), padded prompts,
both extraction modes and the reference's fixed 512-token length."""
import ctypes as C

import numpy as np
import pytest

import psnr_util as pu
from gpu_util import rel_l2
from oracle import model_gen as mg
from oracle import qwen3_oracle as qo
from test_qwen3_oracle import CFG, SEED, prompt

pytestmark = pytest.mark.gpu

TOL = 1e-2       # rows of real tokens
TOL_ALL = 1.5e-2  # every row, padded ones included


def check(got, ref, ntok):
    assert rel_l2(got[:ntok], ref[:ntok]) < TOL, rel_l2(got[:ntok], ref[:ntok])
    assert rel_l2(got, ref) < TOL_ALL, rel_l2(got, ref)


@pytest.fixture(scope="module")
def enc(iris, tmp_path_factory):
    d = mg.make_qwen3_model(str(tmp_path_factory.mktemp("q3gpu")), CFG, SEED)
    m = iris.Qwen3.load(d)
    yield m, d, mg.qwen3_weights(CFG, SEED)
    m.close()


@pytest.mark.parametrize("seq,ntok", [(64, 40), (200, 200), (512, 77)])
def test_flux_extraction_matches_oracle(enc, seq, ntok):
    m, _, w = enc
    m.set_extraction_mode(0)
    ids, mask = prompt(seq, ntok, seed=seq)
    got = m.forward(ids, mask)
    ref = qo.forward(w, CFG, ids, mask)
    assert got.shape == ref.shape == (seq, 3 * CFG["hidden_size"])
    assert np.isfinite(got).all()
    # each extracted layer separately (8, 17, 26)
    H = CFG["hidden_size"]
    for j in range(3):
        check(got[:, j * H:(j + 1) * H], ref[:, j * H:(j + 1) * H], ntok)


def test_zimage_extraction_matches_oracle(enc):
    m, _, w = enc
    m.set_extraction_mode(1)
    ids, mask = prompt(96, 60, seed=9)
    got = m.forward(ids, mask)
    ref = qo.forward(w, CFG, ids, mask, zimage=True)
    m.set_extraction_mode(0)
    assert got.shape == (96, CFG["hidden_size"])
    check(got, ref, 60)


def test_matches_reference_encoder(enc):
    m, d, _ = enc
    ref = pu.ref_lib_or_skip()
    m.set_extraction_mode(0)
    ids, mask = prompt(512, 77, seed=21)
    a = m.forward(ids, mask)
    b = ref.qwen3_forward(d, ids, mask, 3 * CFG["hidden_size"])
    check(a, b, 77)


def test_causal_rows_ignore_later_tokens_and_replay(enc):
    m, _, _ = enc
    m.set_extraction_mode(0)
    ids, mask = prompt(160, 160, seed=4)
    a = m.forward(ids, mask)
    assert np.array_equal(m.forward(ids, mask), a)  # graph replay is deterministic
    ids2 = ids.copy()
    ids2[130:] = (ids2[130:] + 11) % CFG["vocab_size"]
    b = m.forward(ids2, mask)
    # rows 0..127 share query tiles with no changed key: bit-identical
    np.testing.assert_array_equal(a[:128], b[:128])
    assert np.abs(a[130:] - b[130:]).max() > 0.1


def test_device_entry_point_and_errors(iris, enc):
    import torch
    m, _, _ = enc
    m.set_extraction_mode(0)
    ids, mask = prompt(64, 50, seed=8)
    host = m.forward(ids, mask)
    out = torch.zeros(64 * m.text_dim(), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ip = C.POINTER(C.c_int)
    rc = iris.lib().iris_cuda_qwen3_forward_dev(m.h, ids.ctypes.data_as(ip), mask.ctypes.data_as(ip), 64,
                                                C.c_void_p(out.data_ptr()))
    assert rc == 0, iris.last_error()
    assert iris.lib().iris_cuda_synchronize() == 0
    assert np.array_equal(out.cpu().numpy().reshape(64, -1), host)
    big = np.zeros(600, np.int32)
    assert not iris.lib().iris_cuda_qwen3_forward(m.h, big.ctypes.data_as(ip), None, 600)
    assert "sequence length" in iris.last_error()
    with pytest.raises(iris.IrisCudaError):
        m.set_extraction_mode(2)
