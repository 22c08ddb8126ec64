"""Oracle for signs, packing, quantized projections and binary feed-forward blocks.

Test infrastructure only (see ``oracle/__init__.py``).  All arithmetic is
float32 with numpy's IEEE-754 round-to-nearest operations, one operation at a
time, so the order written here is the order the CUDA kernels follow.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _f32(value) -> np.ndarray:
    return np.asarray(value, dtype=np.float32)


# --------------------------------------------------------------------------- signs


def hard_sign(latent: np.ndarray) -> np.ndarray:
    """``w >= 0 -> +1.0`` else ``-1.0`` (so ``-0.0 -> +1``).

    Follows ``w1a1_eagle/model.py:66-68`` (``sign_forward``) and the F32 check of
    ``hard_sign`` at ``model.py:92-95``.
    """
    latent = np.asarray(latent)
    if latent.dtype != np.float32:
        raise ValueError("latent signs must be F32")
    return np.where(latent >= 0, F32(1.0), F32(-1.0)).astype(np.float32)


def sign_backward(grad: np.ndarray, latent: np.ndarray, window: float = 1.0) -> np.ndarray:
    """Straight-through gradient ``grad * 1[|w| <= window]``, inclusive at the edge.

    ``model.py:71-73`` uses window 1.0; a learned/fixed clip window alpha replaces
    the constant for the clipped-STE variant.
    """
    grad = _f32(grad)
    mask = (np.abs(_f32(latent)) <= F32(window)).astype(np.float32)
    return (grad * mask).astype(np.float32)


def packed_signs(latent: np.ndarray) -> np.ndarray:
    """GGUF sign words: bit ``j`` of word ``w`` of row ``r`` is ``latent[r, 32w + j] >= 0``.

    Rows are padded with zero bits to a multiple of 32 columns; the result is an
    int32 ``[rows, ceil(cols / 32)]`` array in little-endian bit order.  Follows
    ``w1a1_eagle/numerical/export.py:79-86`` including its ValueError for a
    non-F32, non-2-D or non-finite input.
    """
    latent = np.asarray(latent)
    if latent.dtype != np.float32 or latent.ndim != 2 or not np.isfinite(latent).all():
        raise ValueError("finite F32 sign matrix required")
    rows, cols = latent.shape
    words = (cols + 31) // 32
    bits = np.zeros((rows, words * 32), dtype=np.uint8)
    bits[:, :cols] = latent >= 0
    weights = (np.uint64(1) << np.arange(32, dtype=np.uint64)).astype(np.uint64)
    packed = (bits.reshape(rows, words, 32).astype(np.uint64) * weights).sum(-1)
    return packed.astype(np.uint32).view(np.int32)


# --------------------------------------------------------------------------- tiled layout
#
# The decode kernels read signs in a tiled order ("T16") chosen so that each
# lane of a warp fetches, with one 16-byte load, exactly the bits of its
# m16n8k32 integer-MMA A fragments for 256 columns of two rows:
#   * rows are padded to a multiple of 16, columns to a multiple of 256;
#   * a unit is (row block rb of 16 rows, column pair cp of 256 columns), 512
#     bytes, stored unit after unit with cp fastest;
#   * inside a unit, word ``4 * lane + w`` (lane 0..31, w 0..3) belongs to
#     row ``16 rb + (lane >> 2) + 8 (w & 1)`` and column chunk
#     ``c0 = 256 cp + 128 (w >> 1)``;
#   * bit ``8 j + s`` of that word (s 0..7, j 0..3) is the sign bit of column
#     ``c0 + 32 (s >> 1) + 16 (s & 1) + 4 (lane & 3) + j``.
# A set bit means ``latent >= 0`` exactly as in the GGUF words.


def t16_shape(rows: int, cols: int) -> tuple[int, int]:
    """(row blocks, column pairs) of the T16 layout."""
    return (rows + 15) // 16, (cols + 255) // 256


def t16_index(rows: int, cols: int):
    """Row and column index arrays ``[rb, cp, lane, w, s, j]`` of the T16 layout."""
    nrb, ncp = t16_shape(rows, cols)
    rb = np.arange(nrb)[:, None, None, None, None, None]
    cp = np.arange(ncp)[None, :, None, None, None, None]
    lane = np.arange(32)[None, None, :, None, None, None]
    w = np.arange(4)[None, None, None, :, None, None]
    s = np.arange(8)[None, None, None, None, :, None]
    j = np.arange(4)[None, None, None, None, None, :]
    row = rb * 16 + (lane >> 2) + 8 * (w & 1)
    col = cp * 256 + 128 * (w >> 1) + 32 * (s >> 1) + 16 * (s & 1) + 4 * (lane & 3) + j
    return row, col


def tile_signs_t16(latent: np.ndarray) -> np.ndarray:
    """T16 sign words (uint32, flat) of an F32 ``[rows, cols]`` latent matrix."""
    latent = np.asarray(latent, dtype=np.float32)
    rows, cols = latent.shape
    nrb, ncp = t16_shape(rows, cols)
    bits = np.zeros((nrb * 16, ncp * 256), dtype=np.uint32)
    bits[:rows, :cols] = latent >= 0
    row, col = t16_index(rows, cols)
    out = np.zeros((nrb, ncp, 32, 4), dtype=np.uint32)
    # gather one row block at a time to bound memory
    for b in range(nrb):
        picked = bits[row[b : b + 1], col]  # [1, ncp, 32, 4, 8, 4]
        shift = (8 * np.arange(4)[None, :] + np.arange(8)[:, None]).astype(np.uint32)  # [s, j]
        out[b] = (picked[0] << shift).sum(axis=(-1, -2), dtype=np.uint64).astype(np.uint32)
    return out.reshape(-1)


def untile_signs_t16(words: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of :func:`tile_signs_t16`: boolean ``[rows, cols]`` sign bits."""
    nrb, ncp = t16_shape(rows, cols)
    words = np.asarray(words, dtype=np.uint32).reshape(nrb, ncp, 32, 4)
    row, col = t16_index(rows, cols)
    shift = (8 * np.arange(4)[None, :] + np.arange(8)[:, None]).astype(np.uint32)
    bits = (words[..., None, None] >> shift) & 1  # [nrb, ncp, 32, 4, 8, 4]
    full = np.zeros((nrb * 16, ncp * 256), dtype=bool)
    full[row, col] = bits.astype(bool)
    return full[:rows, :cols]


# --------------------------------------------------------------------------- F8 code layout
#
# Activation codes feed the integer MMAs as B fragments.  The F8 layout stores
# them so that each lane of a warp fetches the fragments of two 32-column
# k-steps with one 16-byte load: blocks of 8 rows by 64 columns (512 bytes),
# row-block major; inside a block, lane ``4 g + q`` (row ``8 nt + g``) holds, for
# k-step ``s`` of the block, the codes of columns ``32 s + 16 h + 4 q + j`` at
# byte ``8 (s & 1) + 4 h + j``.  The row stride ``ld`` is the column count
# rounded up to 256.


def codes_ld(cols: int) -> int:
    return (cols + 255) // 256 * 256


def f8_offsets(rows: int, cols: int) -> np.ndarray:
    """Byte offset of every (row, column) code in the F8 layout, ``[rows, cols]``."""
    ld = codes_ld(cols)
    nsp = ld // 64
    t = np.arange(rows)[:, None]
    k = np.arange(cols)[None, :]
    nt, g = t >> 3, t & 7
    s, kk = k >> 5, k & 31
    half, q, j = kk >> 4, (kk & 15) >> 2, kk & 3
    return (((nt * nsp + (s >> 1)) * 32 + g * 4 + q) << 4) + ((s & 1) << 3) + (half << 2) + j


def f8_bytes(rows: int, cols: int) -> int:
    return (rows + 7) // 8 * 8 * codes_ld(cols)


def tile_codes_f8(codes: np.ndarray) -> np.ndarray:
    """int8 F8 buffer of integer codes ``[rows, cols]`` (padding left zero)."""
    rows, cols = codes.shape
    out = np.zeros(f8_bytes(rows, cols), dtype=np.int8)
    out[f8_offsets(rows, cols)] = codes.astype(np.int8)
    return out


def untile_codes_f8(buffer: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return np.asarray(buffer, dtype=np.int8)[f8_offsets(rows, cols)]


def c16_offsets(rows: int, cols: int, mtiles: int) -> np.ndarray:
    """Byte offset of every (token, column) code in the C16 layout, ``[rows, cols]``.

    C16 holds codes as int8 m16n8k32 A fragments with the tokens on the M side:
    ``[k-step s = k // 32][m-tile][lane][16 bytes]``; lane ``4 (r % 8) + (kk % 16) // 4``
    of token ``16 m + r`` holds register ``r // 8 + 2 (kk // 16)``, byte ``kk % 4``.
    """
    t = np.arange(rows)[:, None]
    k = np.arange(cols)[None, :]
    s, kk = k >> 5, k & 31
    r, m = t & 15, t >> 4
    lane = ((r & 7) << 2) + ((kk & 15) >> 2)
    reg = (r >> 3) + ((kk >> 4) << 1)
    return (((s * mtiles + m) * 32 + lane) << 4) + (reg << 2) + (kk & 3)


def tile_codes_c16(codes: np.ndarray) -> np.ndarray:
    """int8 C16 buffer of integer codes ``[tokens <= 32, cols]`` (padding zero)."""
    rows, cols = codes.shape
    mt = (rows + 15) // 16
    out = np.zeros(codes_ld(cols) // 32 * mt * 512, dtype=np.int8)
    out[c16_offsets(rows, cols, mt)] = codes.astype(np.int8)
    return out


def tile_signs_w8(latent: np.ndarray, stride: int = 1, offset: int = 0) -> np.ndarray:
    """W8 sign words ``[n-tile][group][lane][4 words]`` (uint32) of an F32 matrix.

    Lane ``4 g + t`` of n-tile ``n`` and 128-column word ``w`` (stored as word
    ``w % 4`` of group ``w // 4``): bit ``8 j + 2 ks + r`` is
    ``latent[8 n + g, 128 w + 32 ks + 16 r + 4 t + j] >= 0`` (0 past the matrix).
    ``stride``/``offset`` interleave the n-tiles of several matrices.
    """
    latent = _f32(latent)
    rows, cols = latent.shape
    nt, ng = (rows + 7) // 8, ((cols + 127) // 128 + 3) // 4
    nw = ng * 4
    bits = np.zeros((nt * 8, nw * 128), dtype=np.uint64)
    bits[:rows, :cols] = latent >= 0
    b = bits.reshape(nt, 8, nw, 4, 2, 4, 4)  # n, g, w, ks, r, t, j
    ks, r, j = np.meshgrid(np.arange(4), np.arange(2), np.arange(4), indexing="ij")
    shifts = (8 * j + 2 * ks + r).astype(np.uint64)  # [ks, r, j]
    ordered = b.transpose(0, 2, 1, 5, 3, 4, 6)  # n, w, g, t, ks, r, j
    words = (ordered << shifts).sum(axis=(4, 5, 6)).astype(np.uint32).reshape(nt, ng, 4, 32)
    words = words.transpose(0, 1, 3, 2)  # n, group, lane, word-in-group
    out = np.zeros((nt * stride, ng, 32, 4), dtype=np.uint32)
    out[offset::stride] = words
    return out.reshape(-1)


def tile_signs_d8(latent: np.ndarray) -> np.ndarray:
    """D8 sign bytes ``[n-tile][4-k-step group][lane][4]`` (uint8) of an F32 ``[rows, cols]`` matrix.

    Byte ``s % 4`` of lane ``4 g + t`` at (n-tile ``n``, group ``s // 4``): bit
    ``4 r + j`` is ``latent[8 n + g, 32 s + 16 r + 4 t + j] >= 0`` (0 past the
    matrix); the m16n8k32 B register ``r`` of that n-tile and k-step is nibble
    ``r`` spread to one bit per byte.
    """
    latent = _f32(latent)
    rows, cols = latent.shape
    nt, ksteps = (rows + 7) // 8, (cols + 31) // 32
    g4 = (ksteps + 3) // 4
    bits = np.zeros((nt * 8, g4 * 4 * 32), dtype=np.uint8)
    bits[:rows, :cols] = latent >= 0
    b = bits.reshape(nt, 8, g4, 4, 2, 4, 4)  # n, g, group, q, r, t, j
    r, j = np.meshgrid(np.arange(2), np.arange(4), indexing="ij")
    shifts = (4 * r + j).astype(np.uint8)  # [r, j]
    ordered = b.transpose(0, 2, 1, 5, 3, 4, 6)  # n, group, g, t, q, r, j
    out = (ordered << shifts).sum(axis=(5, 6)).astype(np.uint8)  # n, group, g, t, q
    return out.reshape(-1)


# --------------------------------------------------------------------------- quantizer


def quantize_codes(value: np.ndarray, gain: np.ndarray, bound, bits: int):
    """Learned-gain/clip activation quantizer of ``Projection.forward``.

    ``model.py:128-140``: ``gained = x * exp(log_gain)``; ``bound = exp(log_clip)``;
    ``clipped = max(min(gained, bound), -bound)``; ``normalized = clipped * (max /
    bound)``; ``rounded = round_half_even(normalized).clamp(-max, max)``;
    ``step = bound / max``.  ``gain`` and ``bound`` are the already
    exponentiated F32 values.  ``max / bound`` is evaluated the way torch
    evaluates ``int / tensor``: ``reciprocal(bound) * max`` (two roundings).
    Returns ``(codes, step)``; codes are F32 integers in ``[-max, max]``.
    """
    if bits not in (4, 8):
        raise ValueError("invalid HE4 projection")
    value = _f32(value)
    gain = _f32(gain)
    bound = F32(bound)
    gained = value * gain
    if not np.isfinite(gained).all():
        raise ValueError("nonfinite quantizer input")
    if not np.isfinite(bound) or not bound > 0:
        raise ValueError("invalid learned clipping bound")
    maximum = F32((1 << (bits - 1)) - 1)
    clipped = np.maximum(np.minimum(gained, bound), -bound)
    ratio = (F32(1.0) / bound) * maximum
    normalized = clipped * ratio
    rounded = np.clip(np.rint(normalized), -maximum, maximum).astype(np.float32)
    step = F32(bound / maximum)
    return rounded, step


def integer_dot(codes: np.ndarray, bits_pm: np.ndarray) -> np.ndarray:
    """Exact ``codes @ signs.T`` for integer codes and +-1 signs (int64).

    Evaluated in float64 BLAS: every product and partial sum is an integer of
    magnitude below 2^53, so the result is exact.
    """
    return np.rint(codes.astype(np.float64) @ bits_pm.astype(np.float64).T).astype(np.int64)


def projection_forward(value, latent, scale, midpoint, gain, bound, bits: int) -> np.ndarray:
    """Forward value of ``Projection.forward`` (``model.py:128-150``).

    ``native = (linear(codes, signs) * clamp_min(scale, 0)) * step
    + (codes.sum(-1) * step) * midpoint``.  The integer dot and the code sum are
    exact, so with identical codes this is bit-exact F32 arithmetic.  The
    straight-through surrogate adds exactly zero to the forward value.
    """
    codes, step = quantize_codes(value, gain, bound, bits)
    signs = hard_sign(_f32(latent))
    dot = integer_dot(codes, signs).astype(np.float32)
    total = codes.astype(np.int64).sum(-1, keepdims=True).astype(np.float32)
    scale_c = np.maximum(_f32(scale), F32(0.0))
    return ((dot * scale_c) * step + (total * step) * _f32(midpoint)).astype(np.float32)


def silu(value: np.ndarray) -> np.ndarray:
    """``x / (1 + exp(-x))`` in F32 (torch ``functional.silu``)."""
    value = _f32(value)
    return (value / (F32(1.0) + np.exp(-value))).astype(np.float32)


def rms(value: np.ndarray, weight: np.ndarray, epsilon: float) -> np.ndarray:
    """``value * rsqrt(mean(value^2) + eps) * weight`` (``model.py:50-51``)."""
    value = _f32(value)
    mean = np.mean(value * value, axis=-1, keepdims=True, dtype=np.float32)
    inv = F32(1.0) / np.sqrt(mean + F32(epsilon))
    return (value * inv * _f32(weight)).astype(np.float32)


def he4_ffn(norm, residual, gate, up, down):
    """HE4 SwiGLU tail of ``Layer.forward`` (``model.py:220-223``).

    ``gate``/``up``/``down`` are dicts with ``latent``, ``scale``, ``midpoint``,
    ``gain`` (exponentiated), ``bound`` (exponentiated); gate/up use 4-bit
    codes and share gain/bound (``model.py:184-187``), down uses 8-bit codes
    (``model.py:188-193``).  Returns ``residual + down(silu(gate(n)) * up(n))``;
    ``residual`` may be None (then only the projection output is returned).
    """
    g = projection_forward(norm, gate["latent"], gate["scale"], gate["midpoint"], gate["gain"], gate["bound"], 4)
    u = projection_forward(norm, up["latent"], up["scale"], up["midpoint"], up["gain"], up["bound"], 4)
    h = (silu(g) * u).astype(np.float32)
    d = projection_forward(h, down["latent"], down["scale"], down["midpoint"], down["gain"], down["bound"], 8)
    return d if residual is None else (_f32(residual) + d).astype(np.float32)


# --------------------------------------------------------------------------- pure W1 (config 1)


def w1_ffn(x, w_gate, w_up, w_down) -> np.ndarray:
    """Pure one-bit-weight SwiGLU with per-row scales ``mean|W|``, fp32 activations.

    The reference has no such module; this is built from its parts: signs from
    ``hard_sign`` (``model.py:92``) and row scales from the ``Projection.scale``
    initialiser ``weight.abs().mean(-1)`` (``model.py:123``), applied as
    ``linear(x, signs) * scale`` (``model.py:143``).
    ``y = (silu(gate) * up) @ sign(Wd).T * sd``.
    """
    x = _f32(x)

    def project(v, w):
        w = _f32(w)
        s = np.abs(w).mean(-1, dtype=np.float32)
        return ((v @ hard_sign(w).T).astype(np.float32) * s).astype(np.float32)

    h = (silu(project(x, w_gate)) * project(x, w_up)).astype(np.float32)
    return project(h, w_down)


# --------------------------------------------------------------------------- W1A1 (config 3)

MEAN_LANES = 256


def fixed_mean_abs(value: np.ndarray) -> np.ndarray:
    """Per-row ``mean(|x|)`` in a fixed F32 summation order.

    Contract shared with the CUDA kernel: lane ``l`` of 256 adds ``|x[l]|,
    |x[l+256]|, ...`` sequentially, then the 256 lane sums are combined by a
    balanced binary tree of adjacent pairs ((0+1)+(2+3))..., then divided by
    the row length.  The reference has no W1A1 code; the export rule string
    ``signed_pm_bound_threshold0_nonnegative_positive_zero_row_scale0``
    (``export.py:145``) and the historical ``w1a1_pack_activations`` kernel
    define the sign rule (x >= 0 -> +1) and the per-token mean scale.
    """
    value = np.abs(_f32(value))
    lead, width = value.shape[:-1], value.shape[-1]
    flat = value.reshape(-1, width)
    rounds = (width + MEAN_LANES - 1) // MEAN_LANES
    padded = np.zeros((flat.shape[0], rounds * MEAN_LANES), dtype=np.float32)
    padded[:, :width] = flat
    padded = padded.reshape(flat.shape[0], rounds, MEAN_LANES)
    acc = np.zeros((flat.shape[0], MEAN_LANES), dtype=np.float32)
    for r in range(rounds):
        acc = (acc + padded[:, r]).astype(np.float32)
    while acc.shape[1] > 1:
        acc = (acc[:, 0::2] + acc[:, 1::2]).astype(np.float32)
    mean = (acc[:, 0] / F32(width)).astype(np.float32)
    return mean.reshape(lead)


def w1a1_projection(x, latent, scale):
    """One W1A1 projection: ``(D * scale[o]) * s[t]`` with ``D = K - 2 popc(xa ^ wa)``.

    Returns ``(out, D, s)``: D is the exact +-1 dot (int64), identical to the
    XNOR-popcount formulation; ``s`` is :func:`fixed_mean_abs` of the rows of x.
    """
    x = _f32(x)
    s = fixed_mean_abs(x)
    xs = np.where(x >= 0, 1.0, -1.0)
    ws = np.where(_f32(latent) >= 0, 1.0, -1.0)
    dot = (xs @ ws.T).astype(np.int64)  # float64 BLAS: +-1 sums below 2^53 are exact
    out = (dot.astype(np.float32) * _f32(scale)) * s[:, None]
    return out.astype(np.float32), dot, s


def w1a1_ffn(x, w_gate, w_up, w_down, s_gate=None, s_up=None, s_down=None):
    """W1A1 SwiGLU: every projection input is re-binarised with its per-row mean|x|.

    Row scales default to ``mean|W|`` (``model.py:123``).  Returns
    ``(y, dots)`` where ``dots`` holds the exact integer dots of the three
    projections for bit-exact popcount checks.
    """
    sg = np.abs(_f32(w_gate)).mean(-1, dtype=np.float32) if s_gate is None else _f32(s_gate)
    su = np.abs(_f32(w_up)).mean(-1, dtype=np.float32) if s_up is None else _f32(s_up)
    sd = np.abs(_f32(w_down)).mean(-1, dtype=np.float32) if s_down is None else _f32(s_down)
    g, dg, _ = w1a1_projection(x, w_gate, sg)
    u, du, _ = w1a1_projection(x, w_up, su)
    h = (silu(g) * u).astype(np.float32)
    y, dd, _ = w1a1_projection(h, w_down, sd)
    return y, {"gate": dg, "up": du, "down": dd, "hidden": h}


def pack_bits_rows(value: np.ndarray) -> np.ndarray:
    """GGUF-style sign words of an F32 matrix without the finiteness check."""
    value = _f32(value)
    rows, cols = value.shape
    words = (cols + 31) // 32
    bits = np.zeros((rows, words * 32), dtype=np.uint64)
    bits[:, :cols] = value >= 0
    weights = np.uint64(1) << np.arange(32, dtype=np.uint64)
    return (bits.reshape(rows, words, 32) * weights).sum(-1).astype(np.uint32)


def popcount_dot(x_words: np.ndarray, w_words: np.ndarray, cols: int) -> np.ndarray:
    """``cols - 2 * popc(xa ^ wa)`` summed over words (padding bits are 0 in both)."""
    xor = x_words[:, None, :] ^ w_words[None, :, :]
    bytes_ = xor.view(np.uint8).reshape(xor.shape[0], xor.shape[1], -1)
    pop = np.unpackbits(bytes_, axis=-1).sum(-1, dtype=np.int64)
    return cols - 2 * pop
