"""CPU restatement of the reference's token sampler (src/sampling.rs) -- TEST INFRASTRUCTURE ONLY.

Used by tests/ as the checker of the device sampler (qne_sampler_*); never by the product path.
Follows src/sampling.rs:
  * Sampler::new            :41-44   state = seed * 0x9E3779B97F4A7C15 | 1 (wrapping)
  * next_f32                :46-53   xorshift64 (13, 7, 17), (x >> 40) / 2^24 in f32
  * try_sample              :58-67   NaN / +inf among allowed tokens, or no finite allowed token,
                                     are errors (raised here as ValueError)
  * sample                  :69-78   the pick joins `seen` when presence_penalty != 0
  * choose                  :80-134  greedy (strict > scan), or top-k by logit, weights
                                     exp((l - top) / T), the shortest prefix holding top_p of their
                                     sum, draw r = u * kept walked down the prefix
and the agent's tool-call bias (agent/src/session.rs:400-404: added to one logit first).
All arithmetic on logits and weights is f32 in the reference's order. The reference selects and
sorts with unstable algorithms, so equal logits have no defined order there; this restatement
(like the device sampler) ranks equal logits by lower token index.
"""
import numpy as np

MASK64 = (1 << 64) - 1


class Sampler:
    def __init__(self, temperature=0.6, top_k=20, top_p=0.95, seed=42, presence_penalty=0.0):
        self.temperature = np.float32(temperature)
        self.top_k = int(top_k)
        self.top_p = np.float32(top_p)
        self.presence_penalty = np.float32(presence_penalty)
        self.state = ((int(seed) * 0x9E3779B97F4A7C15) & MASK64) | 1
        self.seen = set()

    def next_f32(self) -> np.float32:
        x = self.state
        x ^= (x << 13) & MASK64
        x ^= x >> 7
        x ^= (x << 17) & MASK64
        self.state = x
        return np.float32(x >> 40) / np.float32(1 << 24)

    def try_sample(self, logits, mask=None, bias_token=-1, bias=0.0) -> int:
        """mask: bool array of allowed tokens (tokens at or past its length are not allowed)."""
        logits = np.array(logits, dtype=np.float32)
        if bias != 0.0 and 0 <= bias_token < logits.size:
            logits[bias_token] = np.float32(logits[bias_token] + np.float32(bias))
        allowed = self._allowed(logits.size, mask)
        vals = logits[allowed]
        if np.any(np.isnan(vals)) or np.any(vals == np.inf):
            raise ValueError("non-finite model logits")
        if not np.any(np.isfinite(vals)):
            raise ValueError("no finite token is allowed by the sampling mask")
        token = self._choose(logits, allowed, mask is not None)
        if self.presence_penalty != 0:
            self.seen.add(token)
        return token

    @staticmethod
    def _allowed(n, mask):
        if mask is None:
            return np.ones(n, dtype=bool)
        m = np.asarray(mask, dtype=bool)
        out = np.zeros(n, dtype=bool)
        k = min(n, m.size)
        out[:k] = m[:k]
        return out

    def _choose(self, logits, allowed, masked) -> int:
        penalty = np.float32(0) if masked else self.presence_penalty
        adj = logits.copy()
        if penalty != 0 and self.seen:
            idx = np.array(sorted(self.seen), dtype=np.int64)
            idx = idx[idx < adj.size]
            adj[idx] = (adj[idx] - penalty).astype(np.float32)
        cand = np.nonzero(allowed)[0]
        if self.temperature <= 0:
            best_v, best_i = np.float32(-np.inf), 0
            v = adj[cand]
            if cand.size:
                m = v.max()
                if m > best_v:
                    best_i = int(cand[np.nonzero(v == m)[0][0]])
            return best_i
        if cand.size == 0:
            return 0
        v = adj[cand]
        order = np.lexsort((cand, -v.astype(np.float64)))  # logit descending, index ascending
        k = min(max(self.top_k, 1), cand.size)
        top_idx = cand[order[:k]]
        top_val = v[order[:k]]
        t = self.temperature
        top = top_val[0]
        weights = [np.float32(np.exp(np.float32((np.float32(l) - top) / t))) for l in top_val]
        total = np.float32(0)
        for w in weights:
            total = np.float32(total + w)
        kept = np.float32(0)
        n = 0
        for w in weights:
            kept = np.float32(kept + w)
            n += 1
            if kept >= np.float32(self.top_p * total):
                break
        r = np.float32(self.next_f32() * kept)
        for i in range(n):
            r = np.float32(r - weights[i])
            if r <= 0:
                return int(top_idx[i])
        return int(top_idx[n - 1])
