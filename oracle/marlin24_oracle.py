"""CPU oracle for the 2:4 sparse W4A16 GEMM path (Sparse-Marlin layout).

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; it is used by ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` as the checker
and as the timed CPU path.  It is a plain-numpy restatement of the
reference algorithm, written from the reference's behaviour, and pinned
against golden vectors produced by the reference's own Python packers
(``tests/golden/make_golden.py``).

Reference files (paths inside hyeonu453/CSED499II):

* ``kernel_experiments/sparse_marlin/src/test_2_4.py:22-70``  gen_quant4_NT
* ``kernel_experiments/sparse_marlin/src/marlin/__init__.py:242-268``  2:4 perms
* ``kernel_experiments/sparse_marlin/src/marlin/__init__.py:331-388``  Layer_2_4.pack
* ``kernel_experiments/sparse_marlin/src/marlin/_semi_structured_conversions.py:21-48``
  metadata reorder offsets
* ``..._semi_structured_conversions.py:54-179``  dense -> (values, meta)
* ``..._semi_structured_conversions.py:186-283`` (values, meta) -> dense
* ``..._semi_structured_conversions.py:286-314`` mask_creator
* ``kernel_experiments/sparse_marlin/metadata_decode/codec.cu:7-41``  3-bit codec
* ``kernel_experiments/sparse_marlin/decoder_dependency/pair.cuh:27-36``  pair decode

Notation: ``K`` in-features, ``N`` out-features, ``M`` batch rows.  Weights are
``(K, N)`` as in the reference's ``linear.weight.data`` (``test_2_4.py:54``).

Packed format (restated; every index below is checked against the
reference packer by the golden tests):

* ``B``: int32 ``(K/32, 2N)``.  Row ``kk`` covers dense ``k`` in
  ``[32kk, 32kk+32)`` = compressed ``kc`` in ``[16kk, 16kk+16)``.  Column
  word ``128*cc + 16*g + 4*t + j`` (``cc`` = 64-column chunk, ``g`` in 0..7,
  ``t`` in 0..3, ``j`` in 0..3) holds eight 4-bit codes; nibble ``i`` is the
  code of the kept value at out-feature ``n = 64cc + 8g + j + 4*((i>>1)&1)``
  and compressed column ``kc = 16kk + 8*(i&1) + 2t + (i>>2)``.
* ``meta``: int16 ``(N, K/16)`` storage, read as flat int32 words.  Word
  ``kk*N + 64*cc + w`` (``w = 32c + 4a + 2d + h``) holds in its low half
  the 4 nibbles of out-feature ``n = 64cc + 8a + 2c + d`` for dense k in
  ``[32kk + 16h, 32kk + 16h + 16)`` and in its high half those of ``n + 4``.
  Nibble = ``idx0 | idx1 << 2`` (positions of the two kept values).
* ``s``: fp16 ``(K/g, N)`` grouped (columns permuted inside each 8-column
  block by ``(0,4,1,5,2,6,3,7)``) or ``(1, N)`` per-column (natural order).
"""
from __future__ import annotations

import numpy as np

MAXQ = 15
ZERO_POINT = 8

# --------------------------------------------------------------------------
# Quantisation and mask (P1 / P4)
# --------------------------------------------------------------------------


def group_scales(w: np.ndarray, groupsize: int) -> np.ndarray:
    """Per-group absmax scales ``absmax * 2/15`` in fp16.

    Follows ``test_2_4.py:28-33``: the max is taken over each group of
    ``groupsize`` rows of ``w`` (K, N) (the whole K when ``groupsize == -1``)
    and multiplied in fp16 by ``2/15``.
    """
    w = np.asarray(w, dtype=np.float16)
    K, N = w.shape
    g = K if groupsize == -1 else groupsize
    absmax = np.abs(w.reshape(K // g, g, N)).max(axis=1)  # fp16, exact
    # torch: s *= 2 / maxq  (fp16 tensor times python float -> fp16 result,
    # computed in fp32 and rounded once)
    return (absmax.astype(np.float32) * np.float32(2.0 / MAXQ)).astype(np.float16)


def quantize_codes(w: np.ndarray, s: np.ndarray, groupsize: int) -> np.ndarray:
    """Unsigned 4-bit codes ``clamp(round(w/s) + 8, 0, 15)`` (K, N) int32.

    ``w / s`` is an fp16 division (``__init__.py:355``, ``test_2_4.py:34``):
    computed in fp32 and rounded to fp16, then rounded half-to-even.
    """
    w = np.asarray(w, dtype=np.float16)
    K, N = w.shape
    g = K if groupsize == -1 else groupsize
    s_full = np.repeat(np.asarray(s, dtype=np.float16).reshape(-1, N), g, axis=0)
    q = (w.astype(np.float32) / s_full.astype(np.float32)).astype(np.float16)
    codes = np.round(q.astype(np.float32)).astype(np.int32) + ZERO_POINT
    return np.clip(codes, 0, MAXQ)


def dequant_codes(codes: np.ndarray, s: np.ndarray, groupsize: int) -> np.ndarray:
    """fp16 ``(code - 8) * s`` as in ``test_2_4.py:37`` (one fp16 rounding)."""
    K, N = codes.shape
    g = K if groupsize == -1 else groupsize
    s_full = np.repeat(np.asarray(s, dtype=np.float16).reshape(-1, N), g, axis=0)
    v = (codes - ZERO_POINT).astype(np.float16).astype(np.float32)
    return (v * s_full.astype(np.float32)).astype(np.float16)


def mask_2_4(x_nk: np.ndarray) -> np.ndarray:
    """2:4 keep-mask over groups of 4 consecutive entries of each row.

    Restates ``mask_creator`` (``_semi_structured_conversions.py:286-314``):
    the two entries with the smallest ``abs`` value in every group of four
    are dropped.  Ties are broken like a stable ascending sort (lower index
    dropped first), which is what the reference's CPU ``argsort`` does.
    """
    x = np.abs(np.asarray(x_nk)).reshape(-1, 4)
    order = np.argsort(x, axis=1, kind="stable")[:, :2]
    mask = np.ones(x.shape, dtype=bool)
    np.put_along_axis(mask, order, False, axis=1)
    return mask.reshape(np.asarray(x_nk).shape)


# --------------------------------------------------------------------------
# 2:4 compression and metadata (P3)
# --------------------------------------------------------------------------


def nibble_from_flags(m0, m1, m2, m3):
    """Metadata nibble ``idx0 | idx1 << 2`` from the four nonzero flags.

    Same boolean functions as ``_semi_structured_conversions.py:133-141``
    (chosen there with a logic minimiser; they also define the nibble for
    groups with fewer or more than two nonzeros).
    """
    e0 = m0 & m1
    e1 = ~m0 & m1
    e2 = ~m0 & ~m1
    idx0 = e1.astype(np.int32) | (e2.astype(np.int32) << 1)
    idx1 = (e0 | e2 | m3).astype(np.int32) | ((e1 | ~m1).astype(np.int32) << 1)
    return idx0, idx1


def meta_scatter_offsets(n_rows: int, meta_cols: int) -> np.ndarray:
    """Flat int16 destination of logical meta element ``(row, col)``.

    Restates ``_calculate_meta_reordering_scatter_offsets`` for int16 meta
    (``_semi_structured_conversions.py:21-48``): rows are swizzled inside
    64-row groups, 2x2 blocks transposed, and the result stored
    column-major interleaved by 2.
    """
    r = np.arange(n_rows)[:, None]
    c = np.arange(meta_cols)[None, :]
    dst_r = (r // 64) * 64 + (r % 2) * 2 + (r % 8) // 4 + ((r % 4) // 2) * 32 + ((r % 64) // 8) * 4
    dst_r = np.broadcast_to(dst_r, (n_rows, meta_cols)).copy()
    dst_c = np.broadcast_to(c, (n_rows, meta_cols)).copy()
    tr = ((dst_r % 2 == 0) & (dst_c % 2 == 1)).astype(np.int64)
    bl = ((dst_r % 2 == 1) & (dst_c % 2 == 0)).astype(np.int64)
    dst_r += tr - bl
    dst_c -= tr - bl
    return (dst_c // 2) * n_rows * 2 + dst_r * 2 + dst_c % 2


def compress_2_4(dense_nk: np.ndarray):
    """Dense (N, K) int codes -> values (N, K/2) and reordered meta (N, K/16) int16.

    A code of 0 counts as a zero entry, as in the reference (``dense != 0``).
    """
    dense = np.asarray(dense_nk, dtype=np.int32)
    n, k = dense.shape
    if n % 32 or k % 16:
        raise ValueError("compress_2_4 needs N % 32 == 0 and K % 16 == 0")
    d4 = dense.reshape(n, k // 4, 4)
    m = d4 != 0
    idx0, idx1 = nibble_from_flags(m[..., 0], m[..., 1], m[..., 2], m[..., 3])
    v0 = np.take_along_axis(d4, idx0[..., None], axis=-1)[..., 0]
    v1 = np.take_along_axis(d4, idx1[..., None], axis=-1)[..., 0]
    values = np.stack([v0, v1], axis=-1).reshape(n, k // 2)
    nib = (idx0 | (idx1 << 2)).reshape(n, k // 16, 4).astype(np.uint32)
    meta_u = nib[..., 0] | (nib[..., 1] << 4) | (nib[..., 2] << 8) | (nib[..., 3] << 12)
    meta_logical = meta_u.astype(np.uint16).view(np.int16)
    out = np.empty(n * (k // 16), dtype=np.int16)
    out[meta_scatter_offsets(n, k // 16).reshape(-1)] = meta_logical.reshape(-1)
    return values, out.reshape(n, k // 16)


def decompress_2_4(values_nk2: np.ndarray, meta: np.ndarray) -> np.ndarray:
    """Inverse of :func:`compress_2_4` (``_semi_structured_conversions.py:186-283``)."""
    values = np.asarray(values_nk2)
    n, k2 = values.shape
    k = 2 * k2
    flat = np.asarray(meta).reshape(-1)
    logical = flat[meta_scatter_offsets(n, k // 16).reshape(-1)].reshape(n, k // 16)
    lu = logical.view(np.uint16).astype(np.uint32)
    idx = np.stack([(lu >> (2 * b)) & 3 for b in range(8)], axis=-1).reshape(n, k // 4, 2)
    dense = np.zeros((n, k // 4, 4), dtype=values.dtype)
    v = values.reshape(n, k // 4, 2)
    np.put_along_axis(dense, idx[..., 1:2], v[..., 1:2], axis=-1)
    np.put_along_axis(dense, idx[..., 0:1], v[..., 0:1], axis=-1)
    return dense.reshape(n, k)


# --------------------------------------------------------------------------
# Marlin tile permutation and nibble packing (P2)
# --------------------------------------------------------------------------


def _b_axes(K: int, N: int):
    """View shapes relating compressed codes (K/2, N) to ``B`` nibbles.

    Compressed row ``kc = 16kk + 8ia + 2t + ib`` and out-feature
    ``n = 64cc + 8g + 4rh + j`` map to nibble ``i = 4ib + 2rh + ia`` of word
    ``128cc + 16g + 4t + j`` in row ``kk`` of ``B``.  Derived from the
    mma.sp m16n8k32 operand-A fragment: thread ``(g, t)`` of the warp serving
    chunk ``cc`` holds rows ``g`` / ``g+8`` at compressed columns
    ``2t, 2t+1, 8+2t, 9+2t`` of each 16-row sub-tile ``j``, and sub-tile row
    ``g + 8rh`` is out-feature ``8g + j + 4rh``.
    """
    values_view = (K // 32, 2, 4, 2, N // 64, 8, 2, 4)  # kk ia t ib cc g rh j
    to_b = (0, 4, 5, 2, 7, 3, 6, 1)                     # kk cc g t j ib rh ia
    return values_view, to_b


def pack_values(values_kn: np.ndarray) -> np.ndarray:
    """Compressed codes (K/2, N) -> packed ``B`` int32 (K/32, 2N)."""
    kh, N = values_kn.shape
    K = 2 * kh
    view, order = _b_axes(K, N)
    nib = np.asarray(values_kn, dtype=np.uint32).reshape(view).transpose(order)
    nib = (nib.reshape(K // 32, 2 * N, 8) & 0xF).astype(np.uint32)
    q = np.zeros((K // 32, 2 * N), dtype=np.uint32)
    for i in range(8):
        q |= nib[..., i] << np.uint32(4 * i)
    return q.view(np.int32)


def unpack_values(B: np.ndarray, K: int, N: int) -> np.ndarray:
    """Inverse of :func:`pack_values`: packed ``B`` -> codes (K/2, N)."""
    view, order = _b_axes(K, N)
    q = np.asarray(B).view(np.uint32).reshape(K // 32, 2 * N)
    nib = np.stack([(q >> np.uint32(4 * i)) & 0xF for i in range(8)], axis=-1).astype(np.int32)
    b_shape = tuple(view[a] for a in order)
    inv = np.argsort(order)
    return np.ascontiguousarray(nib.reshape(b_shape).transpose(inv)).reshape(K // 2, N)


SCALE_PERM_GROUPED = np.array([8 * i + j for i in range(8) for j in (0, 4, 1, 5, 2, 6, 3, 7)])


def permute_scales(s: np.ndarray, groupsize: int) -> np.ndarray:
    """Scale layout consumed by the kernel (``__init__.py:359-365,374``)."""
    s = np.asarray(s, dtype=np.float16)
    N = s.shape[-1]
    if groupsize == -1:
        return s.reshape(-1, N).copy()
    return s.reshape(-1, 64)[:, SCALE_PERM_GROUPED].reshape(-1, N).copy()


def unpermute_scales(s_packed: np.ndarray, groupsize: int) -> np.ndarray:
    s_packed = np.asarray(s_packed, dtype=np.float16)
    N = s_packed.shape[-1]
    if groupsize == -1:
        return s_packed.copy()
    out = np.empty_like(s_packed.reshape(-1, 64))
    out[:, SCALE_PERM_GROUPED] = s_packed.reshape(-1, 64)
    return out.reshape(-1, N)


def pack_2_4(w: np.ndarray, s: np.ndarray, groupsize: int, mask: np.ndarray | None = None):
    """``Layer_2_4.pack(linear, s, trans=True)`` restated (``__init__.py:331-388``).

    ``w``: fp16 (K, N); ``s``: fp16 (K/g, N) or (1, N).  When ``mask``
    (bool (K, N)) is None the 2:4 mask is built on the biased codes, like
    the reference; an explicit mask packs a pre-pruned weight as-is.
    Returns ``(B, meta, s_packed)``.
    """
    w = np.asarray(w, dtype=np.float16)
    K, N = w.shape
    codes = quantize_codes(w, s, groupsize)
    if mask is None:
        mask = mask_2_4(codes.T).T
    masked_nk = (codes * mask).T
    values_nk, meta = compress_2_4(masked_nk)
    B = pack_values(np.ascontiguousarray(values_nk.T))
    return B, meta, permute_scales(s, groupsize)


def unpack_2_4(B: np.ndarray, meta: np.ndarray, K: int, N: int) -> np.ndarray:
    """Packed ``(B, meta)`` -> dense codes (K, N) with -1 at pruned slots."""
    values_kn = unpack_values(B, K, N)
    marker = values_kn.T + 16  # keep code 0 distinct from "pruned"
    dense_nk = decompress_2_4(marker, meta)
    out = dense_nk.T.astype(np.int32) - 16
    out[dense_nk.T == 0] = -1
    return out


def dequant_2_4(B, meta, s_packed, K: int, N: int, groupsize: int) -> np.ndarray:
    """Packed operator inputs -> the fp16 weight (K, N) the GEMM multiplies by.

    Kept entries are ``(code - 8) * s`` rounded once to fp16 (what the
    kernel's dequant-then-scale computes); pruned entries are 0.
    For ``groupsize == -1`` the scale is returned as a separate factor by
    :func:`gemm_oracle`; here it is applied the same way.
    """
    codes = unpack_2_4(B, meta, K, N)
    s = unpermute_scales(s_packed, groupsize)
    w = dequant_codes(np.where(codes < 0, ZERO_POINT, codes), s, groupsize)
    w[codes < 0] = 0
    return w


def gemm_oracle(A: np.ndarray, B, meta, s_packed, groupsize: int) -> np.ndarray:
    """fp32 ``A @ dequant(W)`` -- the reference's torch oracle
    (``metadata_decode/smoke.py:26``; ``test_2_4.py:81``) computed from
    the packed operator inputs."""
    A = np.asarray(A, dtype=np.float16)
    K = A.shape[1]
    N = np.asarray(s_packed).shape[1]
    W = dequant_2_4(B, meta, s_packed, K, N, groupsize).astype(np.float32)
    return A.astype(np.float32) @ W


# --------------------------------------------------------------------------
# Data generation (P1)
# --------------------------------------------------------------------------


def gen_quant4_nt(N: int, K: int, groupsize: int, rng: np.random.Generator, sigma: float = 1.0):
    """Seeded stand-in for ``gen_quant4_NT`` (``test_2_4.py:22-70``).

    Draws W ~ N(0, sigma) fp16 (K, N), builds group scales, codes and the
    2:4 mask on codes, and packs.  Returns ``(uncompress, B, s_packed,
    meta)`` where ``uncompress`` is the fp16 (K, N) oracle weight
    ``mask * (code - 8) * s``.
    """
    w = (rng.standard_normal((K, N)) * sigma).astype(np.float16)
    s = group_scales(w, groupsize)
    codes = quantize_codes(w, s, groupsize)
    ref = dequant_codes(codes, s, groupsize)
    mask = mask_2_4(codes.T).T
    uncompress = np.where(mask, ref, np.float16(0)).astype(np.float16)
    B, meta, s_packed = pack_2_4(ref, s, groupsize)
    return uncompress, B, s_packed, meta


# --------------------------------------------------------------------------
# 3-bit metadata codec (P11 / P12)
# --------------------------------------------------------------------------

# Code tables of codec.cu:11-13.  "High" encodes the first word of each lane
# pair, "low" the second.  Index = 4-bit 2:4 nibble, value = 3-bit code,
# -1 = illegal nibble.
ENC_HIGH = np.full(16, -1, dtype=np.int32)
ENC_LOW = np.full(16, -1, dtype=np.int32)
for _nib, _c in {0xE: 0, 0xD: 1, 0x8: 2, 0x4: 5, 0x9: 6, 0xC: 7}.items():
    ENC_HIGH[_nib] = _c
for _nib, _c in {0xC: 0, 0xD: 1, 0xE: 2, 0x8: 4, 0x9: 5, 0x4: 6}.items():
    ENC_LOW[_nib] = _c
# Decoder truth tables, including the two unused codes of each table
# (decoder_dependency/pair.cu:11; decoder_dependency/experiment.cu:12).
DEC_HIGH = np.array([0xE, 0xD, 0x8, 0xD, 0x3, 0x4, 0x9, 0xC], dtype=np.uint32)
DEC_LOW = np.array([0xC, 0xD, 0xE, 0xA, 0x8, 0x9, 0x4, 0x0], dtype=np.uint32)
# Earlier 3-bit code of 3bit_encoding/experiment.cu:12,83 (dec(x)).
DEC_3BIT_ENCODING = np.array([0x4, 0x4, 0x9, 0x8, 0xE, 0xE, 0xD, 0xC], dtype=np.uint32)


def _encode_words(words: np.ndarray, table: np.ndarray):
    codes = np.zeros(words.shape, dtype=np.uint64)
    errors = 0
    for i in range(8):
        nib = (words >> np.uint32(4 * i)) & 0xF
        c = table[nib]
        errors += int((c < 0).sum())
        codes |= np.where(c < 0, 0, c).astype(np.uint64) << np.uint64(3 * i)
    return codes, errors


def meta3_pack(meta: np.ndarray):
    """4-bit meta (int16, numel % 128 == 0) -> 3-bit meta int32 (numel*3/8).

    Per 64-word block: lane pair ``p`` in 0..15 packs
    ``first = encH(w[p]) | encL(w[p+32]) << 24`` and
    ``second = encH(w[p+16]) | encL(w[p+48]) << 24`` into planes
    ``X[p] = first[0:32]``, ``Y[p] = first[32:48] | second[0:16] << 16``,
    ``Z[p] = second[16:48]`` (``codec.cu:18-24``).  Returns
    ``(packed, n_illegal_nibbles)``.
    """
    m = np.ascontiguousarray(meta)
    if m.dtype != np.int16 or m.size % 128:
        raise ValueError("expected int16 metadata, multiple of 256 bytes")
    w = m.reshape(-1).view(np.uint32).reshape(-1, 64)
    p = np.arange(16)
    h0, e0 = _encode_words(w[:, p], ENC_HIGH)
    l0, e1 = _encode_words(w[:, p + 32], ENC_LOW)
    h1, e2 = _encode_words(w[:, p + 16], ENC_HIGH)
    l1, e3 = _encode_words(w[:, p + 48], ENC_LOW)
    first = h0 | (l0 << np.uint64(24))
    second = h1 | (l1 << np.uint64(24))
    out = np.empty((w.shape[0], 48), dtype=np.uint32)
    out[:, 0:16] = (first & 0xFFFFFFFF).astype(np.uint32)
    out[:, 16:32] = ((first >> np.uint64(32)) | ((second & 0xFFFF) << np.uint64(16))).astype(np.uint32)
    out[:, 32:48] = (second >> np.uint64(16)).astype(np.uint32)
    return out.reshape(-1).view(np.int32), e0 + e1 + e2 + e3


def decode24(x: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Eight 3-bit codes in bits [0, 24) -> eight nibbles via ``table``."""
    x = np.asarray(x, dtype=np.uint32)
    out = np.zeros(x.shape, dtype=np.uint32)
    for i in range(8):
        out |= table[(x >> np.uint32(3 * i)) & 7] << np.uint32(4 * i)
    return out


def pair_decode(a: np.ndarray, b: np.ndarray, upper: np.ndarray):
    """Two loaded words of a lane -> its two 4-bit metadata words.

    Lanes 0..15 load ``(X, Y)`` and lanes 16..31 load ``(Y, Z)``; the high
    code field is ``first[0:24]`` / ``second[0:24]`` and the low field
    ``first[24:48]`` / ``second[24:48]`` (``pair.cuh:27-36``).
    """
    a = np.asarray(a, dtype=np.uint64)
    b = np.asarray(b, dtype=np.uint64)
    v = a | (b << np.uint64(32))
    hi_in = np.where(upper, v >> np.uint64(16), v) & 0xFFFFFF
    lo_in = np.where(upper, v >> np.uint64(40), v >> np.uint64(24)) & 0xFFFFFF
    return decode24(hi_in.astype(np.uint32), DEC_HIGH), decode24(lo_in.astype(np.uint32), DEC_LOW)


def meta3_unpack(packed: np.ndarray) -> np.ndarray:
    """3-bit meta int32 (numel % 48 == 0) -> 4-bit meta int16 (``codec.cu:25-29``)."""
    x = np.ascontiguousarray(packed).reshape(-1).view(np.uint32)
    if x.size % 48:
        raise ValueError("expected compressed metadata (multiple of 48 words)")
    blk = x.reshape(-1, 48)
    lane = np.arange(32)
    a = blk[:, lane]
    b = blk[:, 16 + lane]
    w0, w1 = pair_decode(a, b, (lane & 16) != 0)
    out = np.empty((blk.shape[0], 64), dtype=np.uint32)
    out[:, 0:32] = w0
    out[:, 32:64] = w1
    return out.reshape(-1).view(np.int16)
