"""The Qwen3 text-encoder oracle (oracle/qwen3_oracle.py) pinned on CPU to the
reference's own encoder (qwen3_model_load + qwen3_forward, iris_qwen3.c:1578,
:1072) compiled from its sources (oracle/_ref): Flux extraction (layers 8, 17,
26 concatenated) and Z-Image extraction (layer n - 2), padded prompts (ids
outside the vocabulary embed as zeros, masked keys), the full 512 length."""
import numpy as np
import pytest

import psnr_util as pu
from oracle import model_gen as mg
from oracle import qwen3_oracle as qo

CFG = dict(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
           vocab_size=1000, num_hidden_layers=28, rope_theta=1000000.0)
SEED = 5


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    ref = pu.ref_lib_or_skip()
    d = mg.make_qwen3_model(str(tmp_path_factory.mktemp("q3")), CFG, SEED)
    return ref, d, mg.qwen3_weights(CFG, SEED)


def prompt(seq, ntok, seed=3, pad_id=151643):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, CFG["vocab_size"], seq).astype(np.int32)
    ids[ntok:] = pad_id
    mask = np.zeros(seq, np.int32)
    mask[:ntok] = 1
    return ids, mask


@pytest.mark.parametrize("seq,ntok,zimage", [(64, 40, False), (48, 48, True), (512, 77, False)])
def test_oracle_matches_reference_encoder(model, seq, ntok, zimage):
    ref, d, w = model
    ids, mask = prompt(seq, ntok)
    td = CFG["hidden_size"] * (1 if zimage else 3)
    a = ref.qwen3_forward(d, ids, mask, td, zimage)
    b = qo.forward(w, CFG, ids, mask, zimage)
    assert a.shape == b.shape == (seq, td)
    assert np.linalg.norm(a - b) / np.linalg.norm(a) < 1e-4


def test_oracle_causal_rows_ignore_later_tokens(model):
    """Causal attention: rows before a change of token ids are unchanged."""
    _, _, w = model
    ids, mask = prompt(32, 32)
    a = qo.forward(w, CFG, ids, mask)
    ids2 = ids.copy()
    ids2[20:] = (ids2[20:] + 7) % CFG["vocab_size"]
    b = qo.forward(w, CFG, ids2, mask)
    np.testing.assert_array_equal(a[:20], b[:20])
    assert np.abs(a[20:] - b[20:]).max() > 0.1
