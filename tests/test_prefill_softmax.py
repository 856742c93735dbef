"""The two-pass softmax of the prefill attention kernel (attention_pf.cu),
restated in numpy and checked against the reference's (CPU only).

The reference (modeling_granite.py:89-112 via llm_mega.py:176-202) computes a
score row, takes the fp32 softmax over all visible keys at once and casts the
probabilities to bf16.  The kernel never holds a whole row: pass 1 walks the
keys in tiles of 64, keeping a running max m and an exp-sum l rescaled by
exp(m_old - m_new) whenever the max grows; pass 2 recomputes each score and
forms p = bf16(exp(s - m) * (1 / l)).  The max is the same value either way,
the sum differs only by fp32 summation order, so p may differ from the
reference's in the last bf16 bit where exp(s - m) / l sits on a rounding
boundary.  Checked: identical maxima, sums within 1e-6 relative, at least
99.9 % of the probabilities bit-identical and the rest one bf16 step apart,
and rows of P V within the tests' attention tolerance."""

import numpy as np
import torch


def _bf16(x):
    return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _reference(s):
    """fp32 softmax over the row, cast to bf16 (torch semantics)."""
    t = torch.from_numpy(s.astype(np.float32))
    return torch.softmax(t, dim=-1).to(torch.bfloat16).float().numpy()


def _two_pass(s, tile=64):
    m = np.float32(-np.inf)
    l = np.float32(0.0)
    for k0 in range(0, s.shape[0], tile):
        t = s[k0:k0 + tile].astype(np.float32)
        nm = np.float32(max(m, t.max()))
        l = np.float32(l * np.exp(np.float32(m - nm)) if np.isfinite(m) else 0.0)
        l = np.float32(l + np.exp((t - nm).astype(np.float32)).astype(np.float32).sum(dtype=np.float32))
        m = nm
    inv = np.float32(1.0) / l
    return _bf16(np.exp((s - m).astype(np.float32)).astype(np.float32) * inv), m, l


def test_two_pass_softmax_matches_reference():
    rng = np.random.default_rng(0)
    same = total = 0
    for row in range(400):
        n = int(rng.integers(1, 1024))  # causal: 1..1023 visible keys
        # scores as the kernel forms them: bf16(bf16(q.k) * 1/128) for q.k of a
        # 128-dim product of N(0, 1) vectors scaled like the reference's activations
        qk = rng.standard_normal(n).astype(np.float32) * np.float32(rng.uniform(1, 400))
        s = _bf16(_bf16(qk) * np.float32(1.0 / 128))
        ref = _reference(s)
        got, m, l = _two_pass(s)
        assert m == s.max()
        l_ref = np.exp((s - s.max()).astype(np.float64)).sum()
        assert abs(float(l) - l_ref) <= 1e-6 * l_ref
        eq = got == ref
        same += int(eq.sum())
        total += n
        diff = np.abs(got - ref)[~eq]
        # one bf16 step at the value's magnitude
        assert np.all(diff <= np.maximum(np.abs(ref[~eq]), 1e-38) * 2.0 ** -7 + 1e-45)
        v = rng.standard_normal((n, 16)).astype(np.float32)
        o_ref, o_got = ref @ v, got @ v
        assert np.abs(o_got - o_ref).max() <= 2.0 ** -6 * max(np.abs(o_ref).max(), 1e-3)
    assert same >= 0.999 * total
