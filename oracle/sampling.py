"""CPU restatement of the sampling step at the LM-head boundary (temperature / top-k / top-p).

TEST INFRASTRUCTURE ONLY (checker for tests/; the product path never imports it).

The megakernel reference decodes greedily; its hook at this boundary is the repetition penalty on the logits before
the argmax (megakernel/kernel.cu:793-795).  The reference's speculative-decoding driver has a CPU sampler chain
(repetition penalty -> top_k -> softmax(logit / temperature) -> top_p -> inverse-CDF draw from std::mt19937_64;
dflash/test/test_dflash.cpp:113-188).  That chain is restated below (reference_chain*) and PINNED draw for draw
against the function itself, cut out of the checkout and compiled (oracle/build_oracle.py: build_ref_sampler) and
through a committed fixture made by it.  The CUDA kernel (luce_megakernel_b200/csrc/sampling.cu) draws with the
Gumbel-max rule from its own counter-based generator, so it cannot agree with the chain draw for draw; it is held
  * token for token to sample() below (the kernel's own definition), and
  * to the chain in what the chain defines independently of the generator: the set of tokens that can be drawn
    (support after top_k and top_p) and their probabilities (tests/test_sampling.py).

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


def nucleus_mask(logits, keep, temperature: float, top_p: float) -> np.ndarray:
    """Of the kept set, in descending logit order, the shortest prefix whose softmax(logit / T) mass reaches top_p (the
    crossing element included, logits equal to it all included); top_p outside (0, 1) cuts nothing."""
    if not (0.0 < top_p < 1.0) or not keep.any():
        return keep
    l = np.asarray(logits, dtype=np.float32)
    inv_t = 1.0 / float(np.float32(temperature))
    idx = np.nonzero(keep)[0]
    z = l[idx].astype(np.float64) * inv_t
    w = np.exp(z - z.max())
    order = np.argsort(-z, kind="stable")
    cum = np.cumsum(w[order])
    target = float(np.float32(top_p)) * w.sum()
    first = int(np.searchsorted(cum, target, side="left"))          # first position with cum >= target
    first = min(first, len(order) - 1)
    cut_value = l[idx][order][first]
    out = np.zeros_like(keep)
    out[idx[l[idx] >= cut_value]] = True
    return out


def sample(logits, temperature: float, top_k: int, seed: int, counter: int, top_p: float = 1.0) -> int:
    l = np.asarray(logits, dtype=np.float32)
    n = l.shape[0]
    greedy = not (temperature > 0.0) or top_k == 1
    if greedy:
        v = np.where(np.isnan(l), -np.inf, l.astype(np.float64))
        return int(np.argmax(v)) if np.isfinite(v).any() or (v > -np.inf).any() else 0
    keep = nucleus_mask(l, kept_mask(l, top_k), temperature, top_p)
    if not keep.any():
        return 0
    u = uniforms(seed, counter, n)
    v = l.astype(np.float64) * (1.0 / float(np.float32(temperature))) - np.log(-np.log(u))
    v = np.where(keep, v, -np.inf)
    return int(np.argmax(v))          # first maximum = lowest index


def distribution(logits, temperature: float, top_k: int, top_p: float = 1.0) -> np.ndarray:
    """softmax(logits / temperature) restricted to the kept set: what sample() draws from."""
    l = np.asarray(logits, dtype=np.float64)
    l32 = np.asarray(logits, dtype=np.float32)
    keep = nucleus_mask(l32, kept_mask(l32, top_k), temperature, top_p)
    z = np.where(keep, l / temperature, -np.inf)
    z -= z.max()
    p = np.exp(z)
    return p / p.sum()


# ---- the reference's sampler chain (dflash/test/test_dflash.cpp:113-188), restated -------------------------------

class MT19937_64:
    """std::mt19937_64 (the generator the reference chain draws from)."""
    NN, MM = 312, 156
    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        mt = [seed & self.MASK]
        for i in range(1, self.NN):
            mt.append((6364136223846793005 * (mt[-1] ^ (mt[-1] >> 62)) + i) & self.MASK)
        self.mt, self.i = mt, self.NN

    def next(self) -> int:
        if self.i >= self.NN:
            mt, NN, MM = self.mt, self.NN, self.MM
            for k in range(NN):
                x = (mt[k] & 0xFFFFFFFF80000000) | (mt[(k + 1) % NN] & 0x7FFFFFFF)
                mt[k] = mt[(k + MM) % NN] ^ (x >> 1) ^ (0xB5026F5AA96619E9 if x & 1 else 0)
            self.i = 0
        x = self.mt[self.i]
        self.i += 1
        x ^= (x >> 29) & 0x5555555555555555
        x ^= (x << 17) & 0x71D67FFFEDA60000
        x ^= (x << 37) & 0xFFF7EEE000000000
        x ^= x >> 43
        return x & self.MASK

    def uniform01(self) -> float:
        """std::uniform_real_distribution<double>(0, 1) of libstdc++: one 64-bit draw converted to double, over 2^64."""
        r = float(self.next()) / 18446744073709551616.0
        return r if r < 1.0 else float(np.nextafter(1.0, 0.0))


def reference_chain(logits, temp: float, top_k: int, top_p: float, rep_pen: float = 1.0, history=(), rep_window: int = 256):
    """Candidates (token ids, descending logit) and probabilities (float32) of the reference chain before the draw
    (test_dflash.cpp:132-181).  Equal logits have no defined order there (std::partial_sort / std::sort): callers
    avoid ties."""
    l = np.asarray(logits, dtype=np.float32).copy()
    vocab = l.shape[0]
    rep = np.float32(rep_pen)
    if rep_pen > 1.0 and len(history):
        win = min(len(history), rep_window)
        for t in set(history[len(history) - win:]):
            l[t] = l[t] / rep if l[t] > 0.0 else l[t] * rep
    order = np.argsort(-l, kind="stable")
    if 0 < top_k < vocab:
        order = order[:top_k]
    inv_t = np.float32(1.0) / max(np.float32(1e-3), np.float32(temp))
    maxv = np.float32(l[order[0]] * inv_t)
    probs = np.exp((l[order] * inv_t - maxv).astype(np.float32)).astype(np.float32)
    Z = 0.0
    for p in probs:
        Z += float(p)
    probs = (probs.astype(np.float64) / Z).astype(np.float32)
    if 0.0 < top_p < 1.0:
        cum, cut = 0.0, len(probs)
        tp = float(np.float32(top_p))
        for i, p in enumerate(probs):
            cum += float(p)
            if cum >= tp:
                cut = i + 1
                break
        probs, order = probs[:cut], order[:cut]
        zz = 0.0
        for p in probs:
            zz += float(p)
        probs = (probs.astype(np.float64) / zz).astype(np.float32)
    return order, probs


def reference_chain_draw(logits, temp, top_k, top_p, rng: MT19937_64, rep_pen=1.0, history=()):
    """The chain's draw (test_dflash.cpp:183-188): inverse CDF over the candidates in descending-logit order."""
    order, probs = reference_chain(logits, temp, top_k, top_p, rep_pen, history)
    r = rng.uniform01()
    acc = 0.0
    for i, p in enumerate(probs):
        acc += float(p)
        if r <= acc:
            return int(order[i])
    return int(order[-1])


def compiled_reference_sampler():
    """ctypes handle of the reference chain compiled from its source (oracle/_ref/libref_sampler.so), or None."""
    import ctypes
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_sampler.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    lib.ref_sample_logits.restype = ctypes.c_int
    return lib


def compiled_reference_draws(lib, logits, temp, top_k, top_p, rep_pen, history, seed, n_draws):
    """n_draws consecutive draws from one generator seeded with `seed`, by the compiled reference function."""
    import ctypes
    l = np.ascontiguousarray(logits, dtype=np.float32)
    h = np.ascontiguousarray(history, dtype=np.int32)
    out = np.zeros(n_draws, dtype=np.int32)
    lib.ref_sample_logits(l.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(l.shape[0]), ctypes.c_float(temp), ctypes.c_float(top_p),
                          ctypes.c_int(top_k), ctypes.c_float(rep_pen), h.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(h.shape[0]),
                          ctypes.c_ulonglong(seed), ctypes.c_int(n_draws), out.ctypes.data_as(ctypes.c_void_p))
    return out
