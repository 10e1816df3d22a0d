"""Coefficient bookkeeping for l-major <-> m-major layouts with m truncation.

l-major ("node") layout: index ``l*l + l + m`` for ``m = -l..l``, ``(L+1)^2`` entries.
m-major ("edge frame") layout, truncated to ``|m| <= mmax``: for ``m = 0`` the entries
``l = 0..L``; then for every ``m = 1..mmax`` first the ``+m`` entries for ``l = m..L`` and then
the ``-m`` entries for ``l = m..L``.  This is the order the SO(2) convolution consumes
(reference ``helm/common/so3.py:15-162``); the reference materialises it as a dense
permutation matrix ``to_m`` and multiplies by it, here it is an index list.
"""

from __future__ import annotations

import torch


class CoefficientMapping(torch.nn.Module):
    def __init__(self, lmax: int, mmax: int):
        super().__init__()
        self.lmax, self.mmax = lmax, mmax
        l_of, m_of, lm_index = [], [], []
        m_size = []
        for m in range(mmax + 1):
            ls = list(range(m, lmax + 1))
            m_size.append(len(ls))
            signs = [1] if m == 0 else [1, -1]
            for s in signs:
                for l in ls:
                    l_of.append(l)
                    m_of.append(s * m)
                    lm_index.append(l * l + l + s * m)
        self.m_size = m_size
        self.res_size = len(lm_index)
        # m-major position k holds l-major coefficient lm_index[k]
        self.register_buffer("m_to_lm", torch.tensor(lm_index, dtype=torch.long), persistent=False)
        self.register_buffer("l_harmonic", torch.tensor(l_of, dtype=torch.long), persistent=False)
        self.register_buffer("m_complex", torch.tensor(m_of, dtype=torch.long), persistent=False)

    @property
    def m_offsets(self) -> list[int]:
        """Start of each |m| block in the m-major layout."""
        off = [0]
        for m, s in enumerate(self.m_size):
            off.append(off[-1] + (s if m == 0 else 2 * s))
        return off

    def gate_expand_index(self) -> torch.Tensor:
        """For m-major entries 1.. (skipping l=0), the gate row (l - 1) that scales them."""
        return (self.l_harmonic[1:] - 1).clone()


def l_expand_index(lmax: int) -> torch.Tensor:
    """l of each l-major coefficient."""
    return torch.cat([torch.full((2 * l + 1,), l, dtype=torch.long) for l in range(lmax + 1)])
