"""Oracle for block-draft acceptance: greedy longest prefix and rejection sampling.

Test infrastructure only (see ``oracle/__init__.py``).

Greedy acceptance restates the reference exactly:
  * ``w1a1_eagle/contracts.py:130-137`` / ``native/verifier-trace.hpp:28-34``:
    argmax with strict ``>``, so the lowest index wins ties; non-finite logits
    are refused;
  * ``benchmarks/verifier.py:107-113``: walk the drafts, emit the target argmax
    at each position, stop at the first mismatch or after an accepted EOG that
    is not the last draft, else emit the bonus argmax.
The output convention follows ``benchmarks/acceptance.py:6-36``: ``emitted =
drafts[:accepted] + [next_token]`` with exactly one target token per round.

Rejection sampling has no implementation in the reference (it lives in the
un-vendored llama.cpp fork; the only in-tree pin is the statistical check of
``native/verifier-test.cpp:43-80`` and the EOG break of
``benchmarks/native.py:19-38``).  This module DEFINES the deterministic
contract the CUDA kernels implement bit for bit:
  * uniforms: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), key = the
    64-bit seed, counter = (request, position, purpose, offset); the uniform
    is ``(x0 >> 8) * 2^-24``;
  * ``e(x)`` for ``x <= 0``: ``x`` is clamped at -86.5, ``k = rint(x log2 e)``
    and ``f = x log2 e - k`` each with one fused rounding, ``2^f`` by a
    degree-5 polynomial with a unit constant term (Horner, fused
    multiply-adds), the result ``p 2^k`` formed exactly on the exponent bits;
  * chunks: a row is cut into chunks of 16384 entries; entry
    ``8 (t + 256 j) + e`` of a chunk is item ``e`` of vector ``j`` of lane
    ``t``; a chunk sum adds each lane's items over ``j`` sequentially (eight
    partial sums, one per ``e``), combines the eight by a balanced tree and
    the 256 lane sums by a balanced tree of adjacent pairs;
  * softmax of a row: chunk ``c`` keeps its max ``m_c`` and ``s_c = sum
    e(l - m_c)``; the row max ``m = max m_c`` and ``S = tree over 32 slots of
    s_c e(m_c - m)``; ``p(j) = e(l_j - m) * rcp(S)`` (correctly rounded
    reciprocal, then one multiply);
  * accept draft ``d`` at position i iff ``u * q(d) < p(d)``; an accepted EOG
    that is not the last draft ends the round (emitted as the round's target
    token);
  * on rejection sample from ``max(0, p - q)`` (from ``p`` when that is zero
    everywhere), after all drafts from the unnormalised ``e(l - m)`` of the
    bonus row, by the inverse-CDF search of :func:`sample_index`.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

CHUNK_LANES = 256
CHUNK_VECTORS = 8
VECTOR_ITEMS = 8
CHUNK = CHUNK_LANES * CHUNK_VECTORS * VECTOR_ITEMS  # 16384 entries
MAX_CHUNKS = 32


# --------------------------------------------------------------------------- bf16


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(value: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even F32 -> bf16 bit patterns (uint16)."""
    value = np.asarray(value, dtype=np.float32)
    u = value.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(value)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


# --------------------------------------------------------------------------- greedy


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """Row argmax, lowest index on ties; ValueError on any non-finite logit."""
    logits = np.asarray(logits, dtype=np.float32)
    if logits.shape[-1] == 0:
        raise ValueError("empty logits")
    if not np.isfinite(logits).all():
        raise ValueError("nonfinite verifier logits")
    return np.argmax(logits, axis=-1).astype(np.int32)


def greedy_prefix(targets, drafts, eog) -> tuple[int, int]:
    """Accepted length and next token for one request (``verifier.py:107-113``)."""
    eog = set(int(v) for v in eog)
    n = len(drafts)
    for index in range(n):
        t = int(targets[index])
        if t != int(drafts[index]) or (t in eog and index + 1 < n):
            return index, t
    return n, int(targets[n])


def accept_greedy(logits: np.ndarray, drafts: np.ndarray, eog=()):
    """Greedy block acceptance for ``logits [B, n+1, V]`` and ``drafts [B, n]``.

    Returns ``(accepted [B] int32, next_token [B] int32, targets [B, n+1] int32)``.
    """
    drafts = np.asarray(drafts)
    if drafts.ndim != 2 or logits.shape[:2] != (drafts.shape[0], drafts.shape[1] + 1):
        raise ValueError("logits must be [requests, drafts + 1, vocab]")
    targets = argmax_rows(logits)
    accepted = np.zeros(drafts.shape[0], dtype=np.int32)
    nxt = np.zeros(drafts.shape[0], dtype=np.int32)
    for b in range(drafts.shape[0]):
        accepted[b], nxt[b] = greedy_prefix(targets[b], drafts[b], eog)
    return accepted, nxt, targets


# --------------------------------------------------------------------------- Philox4x32-10

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint64(0x9E3779B9)
PHILOX_W1 = np.uint64(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(counter: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """Philox4x32 with 10 rounds (Salmon et al., SC'11). ``counter [..., 4]`` uint32."""
    c = [np.asarray(counter[..., i], dtype=np.uint64) for i in range(4)]
    k0 = np.uint64(key[0]) & MASK32
    k1 = np.uint64(key[1]) & MASK32
    for _ in range(10):
        p0 = PHILOX_M0 * c[0]
        p1 = PHILOX_M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK32
        c = [(hi1 ^ c[1] ^ k0) & MASK32, lo1, (hi0 ^ c[3] ^ k1) & MASK32, lo0]
        k0 = (k0 + PHILOX_W0) & MASK32
        k1 = (k1 + PHILOX_W1) & MASK32
    return np.stack(c, axis=-1).astype(np.uint32)


def uniform(seed: int, request: int, position: int, purpose: int, offset: int = 0) -> np.float32:
    """The contract's uniform in [0, 1): ``(x0 >> 8) * 2^-24``."""
    ctr = np.array([request, position, purpose, offset], dtype=np.uint64) & MASK32
    out = philox4x32_10(ctr[None, :], (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return F32(int(out[0, 0]) >> 8) * F32(2.0**-24)


# --------------------------------------------------------------------------- deterministic exp


def _f32(bits: int) -> np.float32:
    return np.array([bits], dtype=np.uint32).view(np.float32)[0]


LOG2E = _f32(0x3FB8AA3B)
ROUND_MAGIC = F32(12582912.0)  # 1.5 * 2^23: adding it rounds to an integer held in the low mantissa bits
EXP_FLOOR = F32(-86.5)         # keeps k >= -125, so p * 2^k stays a normal number
# 2^f ~ 1 + f (c1 + f (c2 + f (c3 + f (c4 + f c5)))) on [-1/2, 1/2]: Chebyshev
# interpolation of (2^f - 1) / f at degree 4, coefficients rounded to F32
EXP2_COEFFS = tuple(_f32(b) for b in (0x3F317218, 0x3E75FD26, 0x3D6357F7, 0x3C1E5FB0, 0x3AAF6433))


def fma32(a, b, c) -> np.ndarray:
    """Correctly rounded F32 fused multiply-add (IEEE 754 ``fusedMultiplyAdd``).

    ``a*b`` is exact in F64; TwoSum gives ``s + err == a*b + c`` exactly; the
    F64 -> F32 rounding of ``s`` is then corrected where ``s`` sits exactly on
    an F32 midpoint and ``err`` says which side the exact value is on.
    """
    a64, b64, c64 = (np.asarray(v, dtype=np.float32).astype(np.float64) for v in (a, b, c))
    ab = a64 * b64
    s = ab + c64
    bb = s - ab
    err = (ab - (s - bb)) + (c64 - bb)
    r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    up = np.nextafter(r, F32(np.inf))
    dn = np.nextafter(r, F32(-np.inf))
    d = s - r64
    mid_up = (d > 0) & (d == (up.astype(np.float64) - r64) / 2) & (err > 0)
    mid_dn = (d < 0) & (-d == (r64 - dn.astype(np.float64)) / 2) & (err < 0)
    return np.where(mid_up, up, np.where(mid_dn, dn, r)).astype(np.float32)


def exp_fixed(x: np.ndarray) -> np.ndarray:
    """The contract's ``e(x)`` for ``x <= 0`` (F32 in, F32 out)."""
    x = np.maximum(np.asarray(x, dtype=np.float32), EXP_FLOOR)
    tm = fma32(x, LOG2E, ROUND_MAGIC)
    kf = (tm - ROUND_MAGIC).astype(np.float32)
    f = fma32(x, LOG2E, -kf)
    p = np.full(f.shape, EXP2_COEFFS[4], dtype=np.float32)
    for c in EXP2_COEFFS[3::-1]:
        p = fma32(p, f, c)
    p = fma32(p, f, F32(1.0))
    bits = p.view(np.uint32) + (tm.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def rcp32(x) -> np.float32:
    """Correctly rounded F32 reciprocal."""
    return F32(1.0) / np.float32(x)


# --------------------------------------------------------------------------- fixed reductions


def chunk_count(vocab: int) -> int:
    return (vocab + CHUNK - 1) // CHUNK


def chunked(values: np.ndarray, fill=0.0) -> np.ndarray:
    """``[..., V] -> [..., C, J, T, E]``: entry ``8 (t + 256 j) + e`` of chunk ``c``.

    A single-chunk row keeps only the vectors and the power-of-two prefix of
    lanes it reaches: the rest hold zero weights, which leave every sum, scan
    and pick of the contract unchanged.
    """
    n = values.shape[-1]
    c = chunk_count(n)
    j_used, t_used = CHUNK_VECTORS, CHUNK_LANES
    if c == 1:
        j_used = -(-n // (CHUNK_LANES * VECTOR_ITEMS))
        if j_used == 1:
            t_used = 1 << max(0, (-(-n // VECTOR_ITEMS) - 1).bit_length())
    padded = np.full(values.shape[:-1] + (c * CHUNK,), fill, dtype=np.float32)
    padded[..., :n] = values
    full = padded.reshape(values.shape[:-1] + (c, CHUNK_VECTORS, CHUNK_LANES, VECTOR_ITEMS))
    return full[..., :j_used, :t_used, :]


def tree_sum(values: np.ndarray) -> np.ndarray:
    """Balanced tree of adjacent pairs over the last axis (a power of two)."""
    acc = np.asarray(values, dtype=np.float32)
    while acc.shape[-1] > 1:
        acc = (acc[..., 0::2] + acc[..., 1::2]).astype(np.float32)
    return acc[..., 0]


def lane_sums(blocks: np.ndarray) -> np.ndarray:
    """``[..., J, T, E] -> [..., T]``: sequential over ``j`` per item, tree over the 8 items."""
    acc = blocks[..., 0, :, :]
    for j in range(1, blocks.shape[-3]):
        acc = (acc + blocks[..., j, :, :]).astype(np.float32)
    return tree_sum(acc)


def chunk_sums(weights: np.ndarray) -> np.ndarray:
    """``[..., V] -> [..., C]`` chunk sums of non-negative weights."""
    return tree_sum(lane_sums(chunked(weights)))


def hs_inclusive(lanes: np.ndarray) -> np.ndarray:
    """Hillis-Steele inclusive scan over the last axis (F32, fixed order)."""
    x = lanes.astype(np.float32).copy()
    d = 1
    while d < x.shape[-1]:
        y = x.copy()
        y[..., d:] = (x[..., d:] + x[..., :-d]).astype(np.float32)
        x = y
        d *= 2
    return x


def sample_index(weights: np.ndarray, u: np.float32) -> int:
    """Inverse-CDF draw from non-negative F32 ``weights`` (one row).

    1. ``run`` = sequential prefix of the chunk sums, ``target = u * run[C]``;
       chunk ``k`` = first with ``run[k] + w_k > target`` (else the last chunk
       with a positive sum, else 0);
    2. lane ``t`` = smallest with ``run[k] + incl[t] > target``, ``incl`` the
       Hillis-Steele inclusive scan of the chunk's lane sums (else the largest
       lane with a positive sum, else 0);
    3. item = first, in the lane's order (vector ``j`` major, item ``e``), with
       ``run[k] + (excl[t] + seq) > target``, ``excl[t] = incl[t-1]`` (0 for
       t = 0) and ``seq`` the lane's sequential prefix (else the last item with
       a positive weight, else the lane's first item).
    """
    weights = np.asarray(weights, dtype=np.float32)
    n = weights.shape[-1]
    sums = chunk_sums(weights)
    run = np.zeros(sums.shape[-1] + 1, dtype=np.float32)
    for c in range(sums.shape[-1]):
        run[c + 1] = F32(run[c] + sums[c])
    target = F32(F32(u) * run[-1])
    hit = np.nonzero((run[:-1] + sums).astype(np.float32) > target)[0]
    if hit.size:
        k = int(hit[0])
    else:
        pos = np.nonzero(sums > 0)[0]
        k = int(pos[-1]) if pos.size else 0
    blocks = chunked(weights)[k]                    # [J, T, E]
    lanes = lane_sums(blocks)
    incl = hs_inclusive(lanes)
    hit = np.nonzero((run[k] + incl).astype(np.float32) > target)[0]
    if hit.size:
        lane = int(hit[0])
    else:
        pos = np.nonzero(lanes > 0)[0]
        lane = int(pos[-1]) if pos.size else 0
    excl = F32(0.0) if lane == 0 else incl[lane - 1]
    items = blocks[:, lane, :].reshape(-1)          # j-major, then e
    chosen, last_pos, acc = -1, -1, F32(0.0)
    for i, w in enumerate(items):
        acc = F32(acc + w) if i else w
        if chosen < 0 and F32(run[k] + F32(excl + acc)) > target:
            chosen = i
        if w > 0:
            last_pos = i
    if chosen < 0:
        chosen = last_pos if last_pos >= 0 else 0
    j, e = divmod(chosen, VECTOR_ITEMS)
    return min(k * CHUNK + VECTOR_ITEMS * (lane + CHUNK_LANES * j) + e, n - 1)


def row_stats(logits_row: np.ndarray):
    """``(m, S)`` of one row under the chunked softmax contract."""
    row = np.asarray(logits_row, dtype=np.float32)
    if not np.isfinite(row).all():
        raise ValueError("nonfinite verifier logits")
    n = row.shape[-1]
    blocks = chunked(row, fill=-np.inf)
    m_c = blocks.reshape(blocks.shape[0], -1).max(axis=1)
    valid = chunked(np.ones(n, np.float32)) > 0
    e = np.where(valid, exp_fixed(np.where(valid, blocks - m_c[:, None, None, None], F32(0.0))), F32(0.0))
    s_c = tree_sum(lane_sums(e.astype(np.float32)))
    m = m_c.max()
    slots = np.zeros(MAX_CHUNKS, np.float32)
    slots[: m_c.shape[0]] = (s_c * exp_fixed((m_c - m).astype(np.float32))).astype(np.float32)
    return F32(m), F32(tree_sum(slots))


def probabilities(row: np.ndarray, m, total) -> np.ndarray:
    """``p(j) = e(l_j - m) * rcp(S)`` for a row (F32)."""
    return (exp_fixed((np.asarray(row, np.float32) - F32(m)).astype(np.float32)) * rcp32(total)).astype(np.float32)


def accept_rejection(target_logits, draft_logits, drafts, seed: int, offset: int = 0, eog=()):
    """Temperature-1 speculative rejection sampling under the contract above.

    ``target_logits [B, n+1, V]``, ``draft_logits [B, n, V]`` (F32 values of
    bf16 inputs), ``drafts [B, n]``.  Returns ``(accepted [B], next_token [B])``.
    """
    target_logits = np.asarray(target_logits, dtype=np.float32)
    draft_logits = np.asarray(draft_logits, dtype=np.float32)
    drafts = np.asarray(drafts)
    B, n = drafts.shape
    if target_logits.shape[:2] != (B, n + 1) or draft_logits.shape[:2] != (B, n):
        raise ValueError("logits must be [requests, drafts + 1, vocab] and [requests, drafts, vocab]")
    if not (np.isfinite(target_logits).all() and np.isfinite(draft_logits).all()):
        raise ValueError("nonfinite verifier logits")
    vocab = target_logits.shape[-1]
    if drafts.size and (drafts.min() < 0 or drafts.max() >= vocab):
        raise ValueError("draft token outside the vocabulary")
    eog = set(int(v) for v in eog)
    accepted = np.zeros(B, dtype=np.int32)
    nxt = np.zeros(B, dtype=np.int32)
    for b in range(B):
        done = False
        for i in range(n):
            mp, sp = row_stats(target_logits[b, i])
            mq, sq = row_stats(draft_logits[b, i])
            d = int(drafts[b, i])
            p = probabilities(target_logits[b, i, d:d + 1], mp, sp)[0]
            q = probabilities(draft_logits[b, i, d:d + 1], mq, sq)[0]
            u = uniform(seed, b, i, 0, offset)
            if F32(u * q) < p:
                if d in eog and i + 1 < n:
                    accepted[b], nxt[b] = i, d
                    done = True
                    break
                continue
            pw = probabilities(target_logits[b, i], mp, sp)
            qw = probabilities(draft_logits[b, i], mq, sq)
            resid = np.maximum((pw - qw).astype(np.float32), F32(0.0))
            if not (resid > 0).any():
                resid = pw
            accepted[b] = i
            nxt[b] = sample_index(resid, uniform(seed, b, i, 1, offset))
            done = True
            break
        if not done:
            mp, _ = row_stats(target_logits[b, n])
            w = exp_fixed((target_logits[b, n] - mp).astype(np.float32))
            accepted[b] = n
            nxt[b] = sample_index(w, uniform(seed, b, n, 1, offset))
    return accepted, nxt
