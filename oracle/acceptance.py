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
contract the CUDA kernel implements bit for bit:
  * uniforms: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), key = the
    64-bit seed, counter = (request, position, purpose, offset); the uniform
    is ``(x0 >> 8) * 2^-24``;
  * ``exp``: Cody-Waite reduction by ln 2 and a degree-7 Taylor polynomial,
    each step a separately rounded F32 multiply or add;
  * softmax sums: tiles of 4096 entries, 512 lanes of 8 contiguous entries;
    each lane adds its 8 sequentially, the 512 lane sums are combined by a
    balanced binary tree of adjacent pairs, tiles are added sequentially;
  * accept draft ``d`` at position i iff ``u * q(d) < p(d)`` with
    ``p = e_p[d] / S_p`` and ``q = e_q[d] / S_q``; an accepted EOG that is
    not the last draft ends the round (emitted as the round's target token);
  * on rejection sample from ``max(0, p - q)``, after all drafts from ``p``
    of the bonus row, by the inverse-CDF search of :func:`sample_index`.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

TILE_LANES = 512
LANE_ITEMS = 8
TILE = TILE_LANES * LANE_ITEMS


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

LOG2E = F32(1.4426950408889634)
# ln 2 split (Cody & Waite): the high part keeps 15 significant bits so that
# k * LN2_HI is exact for |k| <= 2^9; the low part is the F32-rounded rest.
LN2_HI = np.frombuffer(np.array([np.float32(math.log(2.0)).view(np.uint32) & np.uint32(0xFFFFFE00)], dtype=np.uint32).tobytes(), dtype=np.float32)[0]
LN2_LO = F32(math.log(2.0) - float(LN2_HI))
TAYLOR = tuple(F32(1.0 / math.factorial(n)) for n in range(8))  # 1, 1, 1/2, ..., 1/7!


def exp_fixed(x: np.ndarray) -> np.ndarray:
    """Deterministic ``exp`` for ``x <= 0`` (F32, separately rounded steps).

    ``k = rint(x * log2 e)``; ``r = (x - k*LN2_HI) - k*LN2_LO``; Horner of the
    degree-7 Taylor series of ``e^r``; result ``p * 2^k``; 0 for ``k < -126``.
    """
    x = np.asarray(x, dtype=np.float32)
    k = np.rint(x * LOG2E).astype(np.float32)
    r = (x - k * LN2_HI) - k * LN2_LO
    p = TAYLOR[7]
    for n in range(6, -1, -1):
        p = p * r + TAYLOR[n]
    p = np.asarray(p, dtype=np.float32)
    ki = k.astype(np.int64)
    under = ki < -126
    ki = np.clip(ki, -126, 127)
    scale = ((ki + 127).astype(np.uint32) << np.uint32(23)).view(np.float32)
    out = (p * scale).astype(np.float32)
    return np.where(under, F32(0.0), out).astype(np.float32)


# --------------------------------------------------------------------------- fixed reductions


def _tiles(values: np.ndarray) -> np.ndarray:
    n = values.shape[-1]
    ntiles = (n + TILE - 1) // TILE
    padded = np.zeros(values.shape[:-1] + (ntiles * TILE,), dtype=np.float32)
    padded[..., :n] = values
    return padded.reshape(values.shape[:-1] + (ntiles, TILE_LANES, LANE_ITEMS))


def lane_sums(tiles: np.ndarray) -> np.ndarray:
    acc = tiles[..., 0]
    for e in range(1, LANE_ITEMS):
        acc = (acc + tiles[..., e]).astype(np.float32)
    return acc


def tree_sum(lanes: np.ndarray) -> np.ndarray:
    acc = lanes
    while acc.shape[-1] > 1:
        acc = (acc[..., 0::2] + acc[..., 1::2]).astype(np.float32)
    return acc[..., 0]


def tile_total(values: np.ndarray):
    """``(total, tile_sums, running)`` of a row under the fixed tile order."""
    t = _tiles(values)
    sums = tree_sum(lane_sums(t))
    running = np.zeros(sums.shape[:-1] + (sums.shape[-1] + 1,), dtype=np.float32)
    for k in range(sums.shape[-1]):
        running[..., k + 1] = (running[..., k] + sums[..., k]).astype(np.float32)
    return running[..., -1], sums, running


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

    1. ``target = u * total``; tile ``k`` = first with ``running[k] +
       tile_sum[k] > target`` (else the last tile with a positive sum);
    2. lane ``t`` = smallest with ``running[k] + incl[t] > target`` where
       ``incl`` is the Hillis-Steele inclusive scan of the tile's lane sums
       (else the largest lane with a positive sum);
    3. item ``e`` = smallest with ``running[k] + (excl[t] + seq[t][e]) >
       target`` where ``excl[t] = incl[t-1]`` (0 for t = 0) and ``seq`` the
       lane's sequential prefix (else the largest item with a positive
       weight, else item 0 of the lane).
    """
    weights = np.asarray(weights, dtype=np.float32)
    n = weights.shape[-1]
    total, sums, running = tile_total(weights)
    target = F32(u) * total
    t = _tiles(weights)
    hit = np.nonzero((running[:-1] + sums).astype(np.float32) > target)[0]
    if hit.size:
        k = int(hit[0])
    else:
        pos = np.nonzero(sums > 0)[0]
        k = int(pos[-1]) if pos.size else 0
    lanes = lane_sums(t[k])
    incl = hs_inclusive(lanes)
    hit = np.nonzero((running[k] + incl).astype(np.float32) > target)[0]
    if hit.size:
        lane = int(hit[0])
    else:
        pos = np.nonzero(lanes > 0)[0]
        lane = int(pos[-1]) if pos.size else 0
    excl = F32(0.0) if lane == 0 else incl[lane - 1]
    items = t[k, lane]
    seq = np.zeros(LANE_ITEMS, dtype=np.float32)
    acc = F32(0.0)
    for e in range(LANE_ITEMS):
        acc = F32(acc + items[e]) if e else items[0]
        seq[e] = acc
    values = (running[k] + (excl + seq).astype(np.float32)).astype(np.float32)
    hit = np.nonzero(values > target)[0]
    if hit.size:
        item = int(hit[0])
    else:
        pos = np.nonzero(items > 0)[0]
        item = int(pos[-1]) if pos.size else 0
    return min(k * TILE + lane * LANE_ITEMS + item, n - 1)


def row_softmax(logits_row: np.ndarray):
    """``(e, total)``: deterministic unnormalised softmax of one F32 row."""
    row = np.asarray(logits_row, dtype=np.float32)
    if not np.isfinite(row).all():
        raise ValueError("nonfinite verifier logits")
    e = exp_fixed((row - row.max()).astype(np.float32))
    total, _, _ = tile_total(e)
    return e, F32(total)


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
    eog = set(int(v) for v in eog)
    accepted = np.zeros(B, dtype=np.int32)
    nxt = np.zeros(B, dtype=np.int32)
    for b in range(B):
        done = False
        for i in range(n):
            ep, sp = row_softmax(target_logits[b, i])
            eq, sq = row_softmax(draft_logits[b, i])
            d = int(drafts[b, i])
            p = F32(ep[d] / sp)
            q = F32(eq[d] / sq)
            u = uniform(seed, b, i, 0, offset)
            if F32(u * q) < p:
                if d in eog and i + 1 < n:
                    accepted[b], nxt[b] = i, d
                    done = True
                    break
                continue
            pw = (ep / sp).astype(np.float32)
            qw = (eq / sq).astype(np.float32)
            resid = np.maximum((pw - qw).astype(np.float32), F32(0.0))
            if not (resid > 0).any():
                resid = pw
            accepted[b] = i
            nxt[b] = sample_index(resid, uniform(seed, b, i, 1, offset))
            done = True
            break
        if not done:
            ep, _ = row_softmax(target_logits[b, n])
            accepted[b] = n
            nxt[b] = sample_index(ep, uniform(seed, b, n, 1, offset))
    return accepted, nxt
