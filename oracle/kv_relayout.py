"""numpy restatement of the KV append and relayout (test infrastructure only).

Pools are [NB, Hkv, S, 64, 64] (S = D / 64): page (blk, h) is the default stick
tiling of a [64 tokens, D] tile (torch_spyre/csrc/spyre_tensor_impl.cpp:46-175,
device_size [S, 64, 64], stride_map [64, D, 1]).  Everything is a pure copy and
is compared bit-exactly (as int16 bit patterns).

* `append` is the slot write of spyre::overwrite's CPU kernel (narrow + copy_,
  torch_spyre/_inductor/customops.py:298-308) and of index_copy_ into a KV
  cache (tests/inductor/test_inductor_ops.py:5688-5740) at slot = blk*64 + off;
  negative slots are padding and skipped.
* `rows_to_pool` / `pool_to_rows` are the row-major [T, Hkv, D] <-> page
  relayout (token t -> page block_ids[t // 64], row t % 64).
"""

from __future__ import annotations

import numpy as np

PAGE = 64


def _split(rows: np.ndarray) -> np.ndarray:
    """[n, Hkv, D] -> [Hkv, S, n, 64] (page-major order of the same elements)."""
    n, hkv, d = rows.shape
    return rows.reshape(n, hkv, d // 64, 64).transpose(1, 2, 0, 3)


def append(new_rows: np.ndarray, pool: np.ndarray, slots: np.ndarray) -> np.ndarray:
    out = pool.copy()
    nslots = pool.shape[0] * PAGE
    for n, slot in enumerate(slots.tolist()):
        if slot < 0:
            continue
        if slot >= nslots:
            raise IndexError(f"slot {slot} outside the pool ({nslots} slots)")
        blk, t = divmod(slot, PAGE)
        out[blk, :, :, t, :] = new_rows[n].reshape(pool.shape[1], pool.shape[2], 64)
    return out


def rows_to_pool(rows: np.ndarray, pool: np.ndarray, block_ids: np.ndarray) -> np.ndarray:
    out = pool.copy()
    T = rows.shape[0]
    for j in range(-(-T // PAGE)):
        t0, t1 = j * PAGE, min(T, (j + 1) * PAGE)
        out[int(block_ids[j]), :, :, : t1 - t0, :] = _split(rows[t0:t1])
    return out


def pool_to_rows(pool: np.ndarray, block_ids: np.ndarray, T: int) -> np.ndarray:
    hkv, s = pool.shape[1], pool.shape[2]
    rows = np.empty((T, hkv, s * 64), dtype=pool.dtype)
    for j in range(-(-T // PAGE)):
        t0, t1 = j * PAGE, min(T, (j + 1) * PAGE)
        page = pool[int(block_ids[j]), :, :, : t1 - t0, :]      # [Hkv, S, n, 64]
        rows[t0:t1] = page.transpose(2, 0, 1, 3).reshape(t1 - t0, hkv, s * 64)
    return rows
