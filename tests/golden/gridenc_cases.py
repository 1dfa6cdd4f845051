"""Inputs of the hash-grid golden vectors (tests/golden/gridencoder_ref.npz).

Everything here is derived from integer hashing (splitmix64), not from a
random-number library, so the 64 MB hash table that the fixture was made with
is regenerated bit-identically by the tests instead of being stored.

Grid: the benchmark configuration's hash grid -- 16 levels x 2 features, 2^19
rows per level (offsets 2^19 l, gridencoder/grid.py:120-130), base resolution
16, per-level scale 1.447 -- with the parity-stress table U(-1, 1) rounded to
fp16 (the values an fp16 table holds), stored as fp32 as the rasterizer reads
it (hashgrid.h: `const float* hash_features`).
"""
from __future__ import annotations

import numpy as np

LEVELS = 16
LEVEL_DIM = 2
LOG2_T = 19
BASE_RES = 16
PER_LEVEL_SCALE = 1.447
S = np.float32(np.log2(PER_LEVEL_SCALE))  # gridencoder/grid.py:36: S = log2(per_level_scale)
N_FWD = 1024   # points of the forward cases
N_BWD = 128    # points of the backward cases (the first N_BWD of the forward points)
# (align_corners, interpolation 0 linear / 1 smoothstep)
CASES = [(False, 0), (False, 1), (True, 0), (True, 1)]
TABLE_SEED = 0x6E657374
POINT_SEED = 0x706F696E
GRAD_SEED = 0x67726164


def case_name(align: bool, interp: int) -> str:
    return f"a{int(align)}i{interp}"


def offsets() -> np.ndarray:
    return (np.arange(LEVELS + 1, dtype=np.int64) << LOG2_T).astype(np.int32)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def _uniform(n: int, seed: int) -> np.ndarray:
    """n floats in [0, 1) from the top 24 bits of splitmix64(seed * 2^32 + i)."""
    i = np.arange(n, dtype=np.uint64) + (np.uint64(seed) << np.uint64(32))
    return (_splitmix64(i) >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)


def table() -> np.ndarray:
    """[16 * 2^19, 2] fp32 holding fp16 values of U(-1, 1)."""
    rows = LEVELS << LOG2_T
    u = _uniform(rows * LEVEL_DIM, TABLE_SEED)
    return (u * 2 - 1).astype(np.float16).astype(np.float32).reshape(rows, LEVEL_DIM)


def points() -> np.ndarray:
    """[N_FWD, 3] lookup points in [0, 1]^3, with edge cases first: the box
    corners and faces (0 and 1 exactly), points just outside the box (zero
    output, no gradient: gridencoder.cu:108-126, 272-276) and points on cell
    boundaries of the coarse levels."""
    p = _uniform(N_FWD * 3, POINT_SEED).reshape(N_FWD, 3)
    special = np.array([
        [0.0, 0.0, 0.0], [1.0, 1.0, 1.0], [0.5, 0.5, 0.5], [1.0, 0.0, 0.25],
        [0.0, 1.0, 0.75], [-1e-3, 0.5, 0.5], [0.5, 1.0 + 1e-3, 0.5], [0.25, 0.5, -0.25],
        [1.0 / 15.0, 2.0 / 15.0, 3.0 / 15.0], [0.5 / 15.0, 1.5 / 15.0, 2.5 / 15.0],
        [1.0 - 2 ** -24, 2 ** -24, 0.5], [0.999, 0.001, 0.333],
    ], dtype=np.float32)
    p[: len(special)] = special
    return np.ascontiguousarray(p)


def grad_outputs() -> np.ndarray:
    """[LEVELS, N_BWD, 2] upstream gradient U(-1, 1) in gridencoder's [L, B, C] layout."""
    u = _uniform(LEVELS * N_BWD * LEVEL_DIM, GRAD_SEED)
    return (u * 2 - 1).astype(np.float32).reshape(LEVELS, N_BWD, LEVEL_DIM)
