"""Host restatement of the device sampler, for the tests: Philox4x32-10
(Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
SC 2011) and Sampler.SampleTopK (internal/llama/sampling.go:103-143) with the
uniform draw taken from Philox instead of Go's math/rand."""
import math

import numpy as np

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    c = [int(v) & _MASK for v in ctr]
    k0, k1 = int(key[0]) & _MASK, int(key[1]) & _MASK
    for _ in range(10):
        p0, p1 = _M0 * c[0], _M1 * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & _MASK, p1 & _MASK, ((p0 >> 32) ^ c[3] ^ k1) & _MASK, p0 & _MASK]
        k0, k1 = (k0 + _W0) & _MASK, (k1 + _W1) & _MASK
    return c


def uniform(seed: int, counter: int) -> float:
    """The device sampler's U in [0, 1): 53 high bits of Philox word 0:1."""
    c = philox4x32_10([counter & _MASK, counter >> 32, 0, 0], [seed & _MASK, (seed >> 32) & _MASK])
    x = (c[0] << 32) | c[1]
    return (x >> 11) * 2.0 ** -53


def sample_topk(ids, logits, temperature: float, seed: int, counter: int) -> int:
    """SampleTopK over (ids, logits) in list order (float64 softmax of
    float32 differences, cumulative pick)."""
    logits = np.asarray(logits, np.float32)
    mx = logits.max()
    inv_t = 1.0 / float(np.float32(temperature))
    e = [math.exp(float(np.float32(l - mx)) * inv_t) for l in logits]
    r = uniform(seed, counter) * sum(e)
    acc = 0.0
    for i, v in enumerate(e):
        acc += v
        if r <= acc:
            return int(ids[i])
    return int(ids[-1])
