"""The BD3-LM sampler's denoising step and the kernel's Philox draw, on the CPU in numpy.

TEST INFRASTRUCTURE ONLY (see the package docstring): the checker for bd3_subs_sample.

Reference files restated here (paths inside tusharsonthalia/diffusion-llm):
  model/modules.py:791-799   log_softmax: x - max, exp, sum, log, difference
  model/subs.py:8-43         SUBS: -1e6 on the [MASK] logit, log_softmax, carry-over rows
  sample/sampler.py:8-34     sample_categorical: argmax(probs / (EPS - log(u + EPS)))
  sample/sampler.py:100-122  q = exp(log_probs).double() * (1 - s/t), q[mask] = s/t, where()
and the kernel's own draw: Philox4x32-10 (Salmon et al., SC 2011) row uniforms and its
inverse CDF over the kernel's element order (thread t, its 8-entry chunks t, t + 512, ...)
with a Hillis-Steele block scan.
"""

from __future__ import annotations

import numpy as np

from oracle.kv_cache import round_to

EPS = 1e-10
NEG_INF = -1e6


def philox4x32_10(ctr: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """Philox4x32-10 of counters ctr (..., 4) uint32 under a 2 x 32-bit key."""
    m0, m1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
    w0, w1 = 0x9E3779B9, 0xBB67AE85
    c = [ctr[..., i].astype(np.uint64) for i in range(4)]
    k0, k1 = key
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = m0 * c[0]
        p1 = m1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
        k0 = (k0 + w0) & 0xFFFFFFFF
        k1 = (k1 + w1) & 0xFFFFFFFF
    return np.stack([x.astype(np.uint32) for x in c], axis=-1)


def row_uniforms(seed: int, offset: int, rows: int) -> np.ndarray:
    """The kernel's one uniform per row: words x, y of Philox4x32-10 at counter (row, offset
    lo, offset hi, 0x5A3) under key = seed, r = (x << 21 | y >> 11) * 2^-53."""
    ctr = np.zeros((rows, 4), dtype=np.uint32)
    ctr[:, 0] = np.arange(rows, dtype=np.uint32)
    ctr[:, 1] = offset & 0xFFFFFFFF
    ctr[:, 2] = (offset >> 32) & 0xFFFFFFFF
    ctr[:, 3] = 0x5A3
    w = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)).astype(np.uint64)
    return ((w[:, 0] << np.uint64(21)) | (w[:, 1] >> np.uint64(11))).astype(np.float64) * 2.0 ** -53


def _hillis_steele(x: list) -> list:
    """Inclusive scan with the shuffle pattern of the kernel (offsets 1, 2, 4, ...; each round
    adds the value `offset` lanes below from before the round)."""
    x = list(x)
    o = 1
    while o < len(x):
        x = [x[i] + x[i - o] if i >= o else x[i] for i in range(len(x))]
        o <<= 1
    return x


def thread_order(V: int, t: int, threads: int = 512, chunk: int = 8) -> list[int]:
    """The entries thread t of the kernel takes, in its order: chunks c = t, t + threads,
    ..., each the `chunk` consecutive entries [chunk * c, chunk * c + chunk) below V."""
    n_chunks = (V + chunk - 1) // chunk
    return [j for c in range(t, n_chunks, threads) for j in range(chunk * c, min(chunk * c + chunk, V))]


def inverse_cdf(q: np.ndarray, r: float, threads: int = 512):
    """The kernel's inverse-CDF draw from one row of weights q (V,) float64 and a uniform r:
    (index, margin) where margin is the distance of r * total to the nearest slice or
    element boundary, relative to total (rounding decides draws closer than ~1e-15)."""
    V = q.shape[0]
    orders = [thread_order(V, t, threads) for t in range(threads)]
    part = [np.float64(0.0)] * threads
    for t in range(threads):
        acc = np.float64(0.0)
        for j in orders[t]:
            acc = acc + q[j]
        part[t] = acc
    warps = threads // 32
    lanes = [_hillis_steele(part[32 * w:32 * w + 32]) for w in range(warps)]
    wscan = _hillis_steele([lanes[w][31] for w in range(warps)])
    incl = [(wscan[w - 1] if w > 0 else np.float64(0.0)) + lanes[w][l]
            for w in range(warps) for l in range(32)]
    excl = [np.float64(0.0)] + incl[:-1]
    total = incl[-1]
    target = np.float64(r) * total
    if target >= total:
        target = np.nextafter(total, 0.0)
    picks, bounds = [], []
    for t in range(threads):
        bounds.append(incl[t])
        if excl[t] <= target < incl[t]:
            local = target - excl[t]
            acc, last_nz, mine = np.float64(0.0), None, None
            for j in orders[t]:
                acc = acc + q[j]
                bounds.append(excl[t] + acc)
                if q[j] > 0:
                    last_nz = j
                if local < acc:
                    mine = j
                    break
            picks.append(mine if mine is not None else last_nz)
    margin = min(abs(float(target - b_)) for b_ in bounds) / float(total)
    return min(picks), margin


def subs_weights(logits: np.ndarray, mask_index: int, t: float, s: float, dtype: str) -> np.ndarray:
    """q (..., V) float64 of a masked row: SUBS log-softmax in `dtype` (one rounding per op,
    the sum accumulated in float64 here and rounded once), exp in `dtype`, times 1 - s/t,
    and s/t at mask_index."""
    r = lambda a: round_to(a, dtype)  # noqa: E731
    x = np.asarray(logits, dtype=np.float32).copy()
    bias = r(np.float32(NEG_INF))
    x[..., mask_index] = r(x[..., mask_index] + bias)
    shifted = r(x - x.max(axis=-1, keepdims=True))
    e = r(np.exp(shifted))
    total = r(e.astype(np.float64).sum(axis=-1, keepdims=True).astype(np.float32))
    lp = r(shifted - r(np.log(total)))
    q = r(np.exp(lp)).astype(np.float64) * (1 - s / t)
    q[..., mask_index] = s / t
    return q


def subs_sample(logits: np.ndarray, xt: np.ndarray, mask_index: int, t: float, s: float,
                u: np.ndarray, dtype: str):
    """The reference's step replayed with its uniforms u (B, S, V): (tokens, margin) with the
    next tokens (B, S) and, per row, the relative gap between the best and second-best q/g
    (rows where it is below ~1e-6 are decided by rounding)."""
    q = subs_weights(logits, mask_index, t, s, dtype)
    g = EPS - np.log(u + EPS)
    score = q / g
    new = np.argmax(score, axis=-1)
    top2 = np.sort(score, axis=-1)[..., -2:]
    margin = (top2[..., 1] - top2[..., 0]) / np.maximum(top2[..., 1], 1e-300)
    keep = xt != mask_index
    margin = np.where(keep, np.inf, margin)
    return np.where(keep, xt, new), margin


def subs_sample_philox(logits: np.ndarray, xt: np.ndarray, mask_index: int, t: float, s: float,
                       seed: int, offset: int, dtype: str):
    """The kernel's production step: inverse-CDF draws with its Philox row uniforms.
    Returns (tokens, margin) as subs_sample."""
    B, S, V = logits.shape
    q = subs_weights(logits, mask_index, t, s, dtype).reshape(B * S, V)
    r = row_uniforms(seed, offset, B * S)
    tokens = xt.reshape(-1).copy()
    margin = np.full(B * S, np.inf)
    for row in range(B * S):
        if tokens[row] == mask_index:
            tokens[row], margin[row] = inverse_cdf(q[row], r[row])
    return tokens.reshape(B, S), margin.reshape(B, S)
