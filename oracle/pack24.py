"""2:4 pruning and packing oracle (numpy, bit-exact reference for the packer).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Reference algorithm
-------------------
* ``prune_n_m`` (reference ``sparse/pruning.py:28-76``): along the last dim,
  in groups of 4, zero the 2 entries of smallest magnitude
  (``topk(2, largest=False)`` on ``|w|``, line 66; mask scatter, lines 67-68).
* Conv weights are pruned in "columnslast" order: ``W.permute(0,2,3,1)``,
  i.e. groups run along C_in inside each (kh, kw) tap
  (reference ``sengine/optimizer.py:499-523`` validate_2_4_pattern reshapes
  ``(K,C,R,S)->(K,R,S,C)``).  The GEMM reduction index is therefore
  ``k = (kh*KW + kw)*C_in + c``, which is also the ``(KH,KW,Cin,F)`` weight
  layout the reference kernels consume (``sengine/cuda_graph_runtime.py:233-236``).

Packed format (this library's own; the reference has no packer)
---------------------------------------------------------------
``values``  fp16 ``[F_pad, K/2]``: per group of 4, the two kept entries in
            ascending index order.  ``F_pad`` = F rounded up to 128 (one
            tensor-core M tile); padding rows are zero.
``meta``    uint32 ``[F_pad/128, K/32, 128]``: one 32-bit word per tensor-memory
            lane per 32-wide K step of the sparse MMA.  Word for lane ``L``:
              bits [0,16)  row ``r0 = 16*(L//16) + L%8``,
              bits [16,32) row ``r0 + 8``,
              covering K positions ``32*j + 16*((L//8)%2) + [0,16)``; each
              16-bit half holds 4 nibbles (one per group of 4, low nibble
              first); a nibble is ``i0 | (i1 << 2)`` with ``i0 < i1`` the kept
              positions.
            Tie rule: a group with fewer than 2 non-zeros keeps its non-zero
            positions and fills with the lowest unused positions
            (all-zero group -> (0,1) -> 0x4).  A group with more than 2
            non-zeros is rejected.
"""
from __future__ import annotations

import numpy as np

M_TILE = 128      # tensor-core M (output channels per tile)
K_STEP = 32       # logical K of one sparse f16 MMA


def prune_2_4(w: np.ndarray) -> np.ndarray:
    """Zero the 2 smallest-|w| entries of every group of 4 along the last dim.

    Restates reference ``sparse/pruning.py:28-76`` (``prune_n_m`` with n=2,
    m=4, padding the last dim to a multiple of 4 with zeros and trimming
    afterwards).  Among equal magnitudes the lower index is pruned first
    (stable sort); the reference's ``topk`` tie order is not specified, so
    fixtures avoid exact ties.
    """
    w = np.asarray(w)
    shape = w.shape
    w2 = w.reshape(-1, shape[-1])
    rows, cols = w2.shape
    pad = (-cols) % 4
    if pad:
        w2 = np.concatenate([w2, np.zeros((rows, pad), w2.dtype)], axis=1)
    g = w2.reshape(rows, -1, 4)
    order = np.argsort(np.abs(g), axis=2, kind="stable")
    mask = np.ones_like(g)
    np.put_along_axis(mask, order[:, :, :2], 0, axis=2)
    out = (g * mask).reshape(rows, -1)
    if pad:
        out = out[:, :cols]
    return out.reshape(shape)


def prune_conv_weight(w_fchw: np.ndarray) -> np.ndarray:
    """2:4-prune a conv weight ``[F,C,KH,KW]`` along C inside each tap.

    Mirrors the oracle construction ``prune_2_4(W.permute(0,2,3,1))`` then
    permuting back (reference ``sparse/pruning.py:80`` applied in
    ``sengine/optimizer.py:499-523`` order).
    """
    p = prune_2_4(np.transpose(w_fchw, (0, 2, 3, 1)))
    return np.ascontiguousarray(np.transpose(p, (0, 3, 1, 2)))


def verify_2_4(w_fk: np.ndarray) -> bool:
    """Every group of 4 along dim 1 has at least 2 zeros.

    Looser than reference ``verify_n_m`` (``sparse/pruning.py:91-115``),
    which demands exactly 2 zeros; the packer accepts groups with more.
    """
    f, k = w_fk.shape
    g = w_fk[:, : (k // 4) * 4].reshape(f, -1, 4)
    return bool(((g != 0).sum(axis=2) <= 2).all())


def conv_weight_to_fk(w_fchw: np.ndarray, cin_pad: int | None = None) -> np.ndarray:
    """``[F,C,KH,KW]`` -> ``[F, KH*KW*Cp]`` with ``k = (kh*KW+kw)*Cp + c``,
    ``Cp`` = C rounded up to a multiple of 64 (one activation k-block) unless
    ``cin_pad`` says otherwise; the padding columns are zero."""
    f, c = w_fchw.shape[:2]
    cp = cin_pad if cin_pad is not None else -(-c // 64) * 64
    w = np.transpose(w_fchw, (0, 2, 3, 1))
    if cp != c:
        w = np.concatenate([w, np.zeros(w.shape[:3] + (cp - c,), w.dtype)], axis=3)
    return np.ascontiguousarray(w.reshape(f, -1))


def group_indices(w_fk: np.ndarray) -> np.ndarray:
    """Kept index pair ``(i0, i1)`` per group: int ``[F, K/4, 2]``."""
    f, k = w_fk.shape
    if k % 4:
        raise ValueError("K must be a multiple of 4")
    nz = w_fk.reshape(f, k // 4, 4) != 0
    cnt = nz.sum(axis=2)
    if (cnt > 2).any():
        raise ValueError("weight is not 2:4 sparse")
    # Rank positions: non-zeros first (in index order), then zeros (in index
    # order); the first two positions are the kept pair.
    key = np.where(nz, 0, 1) * 4 + np.arange(4)[None, None, :]
    order = np.argsort(key, axis=2, kind="stable")[:, :, :2]
    return np.sort(order, axis=2)


def pack_values(w_fk: np.ndarray, f_pad: int | None = None) -> np.ndarray:
    """Compressed fp16 values ``[F_pad, K/2]`` (kept pair per group)."""
    f, k = w_fk.shape
    if f_pad is None:
        f_pad = -(-f // M_TILE) * M_TILE
    idx = group_indices(w_fk)
    g = w_fk.reshape(f, k // 4, 4).astype(np.float32)
    kept = np.take_along_axis(g, idx, axis=2).reshape(f, k // 2)
    out = np.zeros((f_pad, k // 2), np.float16)
    out[:f] = kept.astype(np.float16)
    return out


def pack_meta(w_fk: np.ndarray, f_pad: int | None = None) -> np.ndarray:
    """Metadata words ``uint32 [F_pad/128, K/32, 128]`` (layout in module doc)."""
    f, k = w_fk.shape
    if k % K_STEP:
        raise ValueError("K must be a multiple of 32")
    if f_pad is None:
        f_pad = -(-f // M_TILE) * M_TILE
    idx = group_indices(w_fk)
    nib = np.full((f_pad, k // 4), 0x4, np.uint32)  # padding rows: (0,1)
    nib[:f] = (idx[:, :, 0] | (idx[:, :, 1] << 2)).astype(np.uint32)
    return _meta_words(nib, f_pad, k)


def _meta_words(nib: np.ndarray, f_pad: int, k: int) -> np.ndarray:
    """Metadata words from one nibble per (row, group of 4) ``[f_pad, k/4]``."""
    n_mt, n_j = f_pad // M_TILE, k // K_STEP
    out = np.zeros((n_mt, n_j, M_TILE), np.uint32)
    lanes = np.arange(M_TILE)
    r0 = 16 * (lanes // 16) + lanes % 8
    half = (lanes // 8) % 2
    for mt in range(n_mt):
        for j in range(n_j):
            g0 = (K_STEP * j + 16 * half) // 4          # first group, per lane
            word = np.zeros(M_TILE, np.uint32)
            for q in range(4):
                word |= nib[mt * M_TILE + r0, g0 + q] << np.uint32(4 * q)
                word |= nib[mt * M_TILE + r0 + 8, g0 + q] << np.uint32(16 + 4 * q)
            out[mt, j] = word
    return out


def unpack(values: np.ndarray, meta: np.ndarray, f: int, k: int) -> np.ndarray:
    """Inverse of the packer: dense ``[f, k]`` float32 from values + meta."""
    f_pad = values.shape[0]
    dense = np.zeros((f_pad, k), np.float32)
    lanes = np.arange(M_TILE)
    r0 = 16 * (lanes // 16) + lanes % 8
    half = (lanes // 8) % 2
    for mt in range(f_pad // M_TILE):
        for j in range(k // K_STEP):
            word = meta[mt, j]
            for hi in (0, 1):
                rows = mt * M_TILE + r0 + 8 * hi
                for q in range(4):
                    nibble = (word >> np.uint32(16 * hi + 4 * q)) & 0xF
                    g = (K_STEP * j + 16 * half) // 4 + q
                    for s, sh in ((0, 0), (1, 2)):
                        pos = (nibble >> sh) & 3
                        dense[rows, 4 * g + pos] = values[rows, 2 * g + s].astype(np.float32)
    return dense[:f]


K_BLOCK = 64      # activation channels per k-block (one 128-byte row of fp16)


def pack_dense_split(w_fchw: np.ndarray):
    """Packed blob parts of a DENSE conv weight ``[F,C,KH,KW]`` run as two
    2:4 halves over the same activations (this library's dense mode; the
    reference keeps such convs unpruned).

    Activation k-block ``kb`` (64 input channels of one tap, ``k = (kh*KW +
    kw)*C + c``) meets weight k-blocks ``2kb`` and ``2kb+1``: in each group of
    four channels the first keeps positions (0,1) (nibble ``0x4``), the second
    positions (2,3) (nibble ``0xE``), whatever the values (zeros included).
    Returns ``(values fp16 [F_pad, K], meta uint32 [F_pad/128, 2K/32, 128])``.
    """
    w_fk = conv_weight_to_fk(w_fchw).astype(np.float32)
    f, k = w_fk.shape
    if k % K_BLOCK:
        raise ValueError("C must be a multiple of 64")
    f_pad = -(-f // M_TILE) * M_TILE
    g = w_fk.reshape(f, k // K_BLOCK, K_BLOCK // 4, 4)          # [f, kb, gi, pos]
    halves = np.stack([g[..., 0:2], g[..., 2:4]], axis=2)      # [f, kb, h, gi, 2]
    vals = np.zeros((f_pad, k), np.float16)
    vals[:f] = halves.reshape(f, k).astype(np.float16)
    nib = np.full((f_pad, 2 * k // 4), 0x4, np.uint32)
    per_block = np.repeat(np.array([0x4, 0xE], np.uint32), K_BLOCK // 4)   # [h*16 + gi]
    nib[:f] = np.tile(per_block, k // K_BLOCK)[None, :]
    return vals, _meta_words(nib, f_pad, 2 * k)
