"""The on-disk formats of the learned path, against files the reference wrote.

tests/golden/ref_codebook_444.npz is a ``prismkv-cb-v1`` codebook saved by the reference's
LearnedSliceCodebook.save (learned_codebook.py:275-323); ref_lloyd_z.npz is a Lloyd-Max z file
saved by its LloydMaxQuantizer1D.save (lloyd_max.py:156-185); files_codes.npz holds seeded
vectors and the codes the reference's quantizer gave after loading each file
(stacked_plane.py:183-204, :349-356).  Reading them here must give the same tables, our files
must carry the keys the reference reads, and the oracle driven by the loaded tables must give
the reference's codes (rounding ties excepted, each proven in fp64).
"""

import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, load_golden
from prismkv_b200 import LearnedSliceCodebook, LloydMaxQuantizer1D
from prismkv_b200.utils import make_rotation

CB = os.path.join(GOLDEN, "ref_codebook_444.npz")
LM = os.path.join(GOLDEN, "ref_lloyd_z.npz")


def test_codebook_file_reads_as_written():
    raw = np.load(CB)
    cb = LearnedSliceCodebook.load(CB)
    assert cb.bins_z == 16 and cb.K == 256
    np.testing.assert_array_equal(cb.codebooks.numpy(), raw["codebooks"])
    assert (cb.z_min, cb.z_max, cb.r_max) == (float(raw["z_min"]), float(raw["z_max"]), float(raw["r_max"]))


def test_codebook_file_round_trips_with_the_reference_keys(tmp_path):
    cb = LearnedSliceCodebook.load(CB)
    out = tmp_path / "cb.npz"
    cb.save(out)
    ours, ref = np.load(out), np.load(CB)
    assert set(ref.files) <= set(ours.files)
    for k in ref.files:
        assert ours[k].dtype == ref[k].dtype and ours[k].shape == ref[k].shape, k
        np.testing.assert_array_equal(ours[k], ref[k])


def test_codebook_file_of_another_version_is_refused(tmp_path):
    raw = dict(np.load(CB))
    raw["version"] = np.bytes_("prismkv-cb-v0")
    bad = tmp_path / "bad.npz"
    np.savez(bad, **raw)
    with pytest.raises(ValueError, match="Unsupported codebook version"):
        LearnedSliceCodebook.load(bad)


def test_lloyd_max_file_reads_as_written(tmp_path):
    raw = np.load(LM)
    lm = LloydMaxQuantizer1D.load(LM)
    np.testing.assert_array_equal(lm.boundaries.numpy(), raw["z_boundaries"])
    np.testing.assert_array_equal(lm.centroids.numpy(), raw["z_centroids"])
    out = tmp_path / "lm.npz"
    lm.save(out)
    ours = np.load(out)
    for k in raw.files:
        np.testing.assert_array_equal(ours[k], raw[k])


@pytest.mark.parametrize("which", ["cb", "lloyd"])
def test_oracle_with_the_loaded_tables_gives_the_reference_codes(which):
    f = load_golden("files_codes")
    R = f["R"]
    np.testing.assert_array_equal(R, make_rotation(96, 42).numpy())
    p = oracle.QuantParams.default(96)
    if which == "cb":
        cb = LearnedSliceCodebook.load(CB)
        p.codebook = cb.codebooks.numpy()
        p.z_min, p.z_max, p.r_max = cb.z_min, cb.z_max, cb.r_max
    else:
        lm = LloydMaxQuantizer1D.load(LM)
        p.lloyd_boundaries = lm.boundaries.numpy()
        p.lloyd_centroids = lm.centroids.numpy()
    ref = f[f"codes_{which}"].astype(np.int64) & 0xFFF
    mine = oracle.encode(f["x"], R, p)
    rep = oracle.classify(f["x"], R, p, mine, ref)
    assert rep.unexplained == 0, rep.examples
