"""The reference's own reproducibility band, used as the whole-forward
tolerance.

The decode step re-quantizes activations to int8 per 32-value block before
every matvec (QuantizeQ8_0Into, q8_0.go:22-79).  Any two correct
implementations whose float32 summation orders differ (the reference's
CGO_ENABLED=1 build with simd.c and its CGO_ENABLED=0 pure-Go build are such
a pair) eventually round some value on opposite sides of a quantization
boundary; that flip perturbs the next stage's inputs, which flips more values,
and the difference saturates at the quantization noise level (about 1% of the
logits) within a few steps.  A float64 implementation of the same algorithm
shows the same band.  The parity bar (logits within 1e-2 relative L2,
greedy ids equal except where the top-2 gap is below 1e-3) is therefore
applied together with this measured band: the GPU may differ from the cgo
reference by no more than the reference's other builds do on the same inputs.
"""
import numpy as np

LOGIT_TOL = 1e-2
GAP_EXEMPT = 1e-3
BAND_MARGIN = 1.5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class ReferenceRuns:
    """Teacher-forced logits of the cgo reference (oracle + simd.c), the pure
    Go reference (oracle restatement only) and, for small models, a float64
    numpy forward, all on the same token ids."""

    def __init__(self, oracle_mod, cfg, T, ids, ctx, with_f64=True, prefix_ids=()):
        import npref
        import synthetic
        self.cgo_model = oracle_mod.OracleModel(cfg, T)
        self.cgo_model.new_state(ctx)
        pure = oracle_mod.OracleModel(cfg, T)
        pure.new_state(ctx)
        f64 = None
        if with_f64:
            factors = synthetic.llama3_freq_factors(cfg) if cfg.rope_scaling else None
            f64 = npref.NpModel(cfg, T, ctx, factors)
        for t in prefix_ids:
            self.cgo_model.forward(int(t), logits=False)
            pure.forward(int(t), logits=False, use_ref=False)
            if f64 is not None:
                f64.forward(int(t))
        self.cgo, self.pure, self.f64 = [], [], []
        for t in ids:
            self.cgo.append(self.cgo_model.forward(int(t)))
            self.pure.append(pure.forward(int(t), use_ref=False))
            if f64 is not None:
                self.f64.append(f64.forward(int(t)).astype(np.float32))
        self.pure_model = pure

    def band(self):
        """Largest relative L2 distance of another reference build from cgo."""
        s = [rel_l2(p, c) for p, c in zip(self.pure, self.cgo)]
        s += [rel_l2(f, c) for f, c in zip(self.f64, self.cgo)]
        return max(s) if s else 0.0

    def tol(self):
        return max(LOGIT_TOL, BAND_MARGIN * self.band())

    def step_noise(self, i):
        """Largest per-logit disagreement between the reference builds at step i."""
        n = float(np.abs(self.pure[i] - self.cgo[i]).max())
        if self.f64:
            n = max(n, float(np.abs(self.f64[i] - self.cgo[i]).max()))
        return n

    def gap_exempt(self, i):
        return max(GAP_EXEMPT, 2.0 * self.step_noise(i))
