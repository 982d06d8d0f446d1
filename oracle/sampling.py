"""CPU restatement of the sampling step at the LM-head boundary (temperature / top-k).

TEST INFRASTRUCTURE ONLY (checker for tests/; the product path never imports it).

The reference decodes greedily; its hook at this boundary is the repetition penalty on the logits before the
argmax (megakernel/kernel.cu:793-795).  parity unpinned: the reference has no sampler to take vectors from; the
CUDA kernel (luce_megakernel_b200/csrc/sampling.cu) is held to this restatement token for token, and this
restatement is held to the softmax distribution it claims to sample from (tests/test_sampling.py).

    kept set = top_k logits by (value descending, index ascending); all of them when top_k <= 0 or >= n
    u_i      = ((splitmix64(seed + counter * 0x9E3779B97F4A7C15 + (i + 1) * 0xD1B54A32D192ED03) >> 11) + 0.5) / 2^53
    token    = argmax over the kept set of logit_i / temperature - log(-log(u_i)), ties to the lowest index
    temperature <= 0 or top_k == 1: the greedy argmax (lowest index on ties).  NaN logits are never chosen.
"""
import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def uniforms(seed: int, counter: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + np.uint64(counter & 0xFFFFFFFFFFFFFFFF) * np.uint64(0x9E3779B97F4A7C15) \
            + i * np.uint64(0xD1B54A32D192ED03)
        z ^= z >> np.uint64(30); z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27); z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) / 9007199254740992.0


def kept_mask(logits: np.ndarray, top_k: int) -> np.ndarray:
    l = np.asarray(logits, dtype=np.float32)
    n = l.shape[0]
    valid = ~np.isnan(l)
    if top_k <= 0 or top_k >= n:
        return valid
    # order: value descending, index ascending; NaN below everything
    key = np.where(valid, l, -np.inf).astype(np.float64)
    order = np.lexsort((np.arange(n), -key))
    keep = np.zeros(n, dtype=bool)
    keep[order[:top_k]] = True
    return keep & valid


def sample(logits, temperature: float, top_k: int, seed: int, counter: int) -> int:
    l = np.asarray(logits, dtype=np.float32)
    n = l.shape[0]
    greedy = not (temperature > 0.0) or top_k == 1
    if greedy:
        v = np.where(np.isnan(l), -np.inf, l.astype(np.float64))
        return int(np.argmax(v)) if np.isfinite(v).any() or (v > -np.inf).any() else 0
    keep = kept_mask(l, top_k)
    if not keep.any():
        return 0
    u = uniforms(seed, counter, n)
    v = l.astype(np.float64) * (1.0 / float(np.float32(temperature))) - np.log(-np.log(u))
    v = np.where(keep, v, -np.inf)
    return int(np.argmax(v))          # first maximum = lowest index


def distribution(logits, temperature: float, top_k: int) -> np.ndarray:
    """softmax(logits / temperature) restricted to the kept set: what sample() draws from."""
    l = np.asarray(logits, dtype=np.float64)
    keep = kept_mask(np.asarray(logits, dtype=np.float32), top_k)
    z = np.where(keep, l / temperature, -np.inf)
    z -= z.max()
    p = np.exp(z)
    return p / p.sum()
