"""On-disk formats of the reference, read and written byte-for-byte.

* ``.fvecs`` / ``.ivecs`` (utils.h:23-94): per row an int32 dimension then the
  row's values.
* ``global_pq_codebook.bin`` (build_global.cu:204-206): raw float32
  ``[pq_m][256][dim/pq_m]``.
* ``ivf_data.bin`` (build_global.cu:242-252; read at search_pipeline.cu:490-503):
  ``int32 total, int32 nlist, int32 offsets[nlist+1], int32 ids[total],
  uint8 codes[total][pq_m], float32 centroids[nlist][dim]``.  The file holds
  neither ``pq_m`` nor ``dim``: the reader infers them from the codebook
  (``pq_m * 256 * sub_dim`` floats) and the file length.
"""
from __future__ import annotations

import os

import numpy as np


def write_vecs(path: str, x: np.ndarray) -> None:
    x = np.ascontiguousarray(x)
    n, d = x.shape
    rec = np.empty((n, 1 + d), dtype=np.int32)
    rec[:, 0] = d
    rec[:, 1:] = x.view(np.int32) if x.dtype.itemsize == 4 else x.astype(np.int32)
    rec.tofile(path)


def read_vecs(path: str, dtype=np.float32) -> np.ndarray:
    raw = np.fromfile(path, dtype=np.int32)
    if raw.size == 0:
        return np.zeros((0, 0), dtype)
    d = int(raw[0])
    rows = raw.reshape(-1, d + 1)
    if not np.all(rows[:, 0] == d):
        raise ValueError(f"{path}: inconsistent row dimensions")
    return np.ascontiguousarray(rows[:, 1:]).view(dtype)


def write_codebook(path: str, codebook: np.ndarray) -> None:
    np.ascontiguousarray(codebook, np.float32).tofile(path)


def read_codebook(path: str, pq_m: int) -> np.ndarray:
    cb = np.fromfile(path, dtype=np.float32)
    if cb.size % (pq_m * 256):
        raise ValueError(f"{path}: {cb.size} floats is not pq_m*256*sub_dim for pq_m={pq_m}")
    return cb.reshape(pq_m, 256, -1)


def write_ivf(path: str, offsets: np.ndarray, ids: np.ndarray, codes: np.ndarray, centroids: np.ndarray) -> None:
    offsets = np.ascontiguousarray(offsets, np.int32)
    ids = np.ascontiguousarray(ids, np.int32)
    codes = np.ascontiguousarray(codes, np.uint8)
    centroids = np.ascontiguousarray(centroids, np.float32)
    nlist = centroids.shape[0]
    assert offsets.shape == (nlist + 1,) and ids.shape[0] == codes.shape[0] == int(offsets[-1])
    with open(path, "wb") as f:
        np.array([ids.shape[0], nlist], np.int32).tofile(f)
        offsets.tofile(f)
        ids.tofile(f)
        codes.tofile(f)
        centroids.tofile(f)


def read_ivf(path: str, pq_m: int, dim: int) -> dict:
    with open(path, "rb") as f:
        total, nlist = (int(v) for v in np.fromfile(f, np.int32, 2))
        offsets = np.fromfile(f, np.int32, nlist + 1)
        ids = np.fromfile(f, np.int32, total)
        codes = np.fromfile(f, np.uint8, total * pq_m).reshape(total, pq_m)
        centroids = np.fromfile(f, np.float32, nlist * dim).reshape(nlist, dim)
    if centroids.size != nlist * dim:
        raise ValueError(f"{path}: truncated (pq_m={pq_m}, dim={dim} do not match the file)")
    return dict(offsets=offsets, ids=ids, codes=codes, centroids=centroids)


def save_index(res_dir: str, index: dict) -> None:
    """Write ``ivf_data.bin`` and ``global_pq_codebook.bin`` into ``res_dir``."""
    os.makedirs(res_dir, exist_ok=True)
    write_codebook(os.path.join(res_dir, "global_pq_codebook.bin"), index["codebook"])
    write_ivf(os.path.join(res_dir, "ivf_data.bin"), index["offsets"], index["ids"], index["codes"],
              index["centroids"])


def load_index(res_dir: str, pq_m: int, dim: int) -> dict:
    cb = read_codebook(os.path.join(res_dir, "global_pq_codebook.bin"), pq_m)
    if cb.shape[2] * pq_m != dim:
        raise ValueError(f"codebook sub_dim {cb.shape[2]} * pq_m {pq_m} != dim {dim}")
    ivf = read_ivf(os.path.join(res_dir, "ivf_data.bin"), pq_m, dim)
    ivf["codebook"] = cb
    return ivf
