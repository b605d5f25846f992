import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


def golden_files(prefix=""):
    return sorted(glob.glob(os.path.join(GOLDEN, f"{prefix}*.npz")))


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name if name.endswith(".npz") else name + ".npz")))


def params_from(f):
    """oracle.QuantParams from a golden fixture's quantizer state."""
    from oracle import QuantParams
    b = f["bits"]
    r = f["ranges"]
    p = QuantParams(dim=int(f["dim"]), bits_z=int(b[0]), bits_r=int(b[1]), bits_theta=int(b[2]),
                    z_min=float(r[0]), z_max=float(r[1]), r_max=float(r[2]))
    if "codebook" in f:
        p.codebook = f["codebook"]
    if "lloyd_boundaries" in f:
        p.lloyd_boundaries = f["lloyd_boundaries"]
        p.lloyd_centroids = f["lloyd_centroids"]
    if "bias_table" in f:
        p.bias_table = f["bias_table"]
        p.bias_delta_z = float(f["bias_delta_z"])
    return p


def quantizer_from(f):
    """prismkv_b200 quantizer with a golden fixture's exact state (rotation included)."""
    import torch
    from prismkv_b200 import StackedPlaneQuantizer, LearnedSliceCodebook, BiasTable, LloydMaxQuantizer1D
    b = [int(x) for x in f["bits"]]
    r = f["ranges"]
    q = StackedPlaneQuantizer.from_rotation(torch.from_numpy(f["R"]), *b, z_min=float(r[0]),
                                            z_max=float(r[1]), r_max=float(r[2]))
    Cz, K = 1 << b[0], 1 << (b[1] + b[2])
    if "codebook" in f:
        q._codebooks = LearnedSliceCodebook(torch.from_numpy(f["codebook"]), Cz, K, q.z_min, q.z_max, q.r_max)
    if "lloyd_boundaries" in f:
        lm = LloydMaxQuantizer1D(K=Cz)
        lm.boundaries = torch.from_numpy(f["lloyd_boundaries"])
        lm.centroids = torch.from_numpy(f["lloyd_centroids"])
        q._lloyd_max_z = lm
    if "bias_table" in f:
        q._bias = BiasTable(torch.from_numpy(f["bias_table"]), delta_z=float(f["bias_delta_z"]))
    return q


@pytest.fixture(scope="session")
def cuda_ready():
    import torch
    from prismkv_b200 import _lib
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    _lib.load()
    return True
