"""Real-basis Wigner 3j tensors and the coupled <-> uncoupled basis transform.

``wigner_3j(l1, l2, l3)`` is the unit-Frobenius-norm tensor ``C[i, j, k]`` that is invariant
under simultaneous rotation, ``C = (D1 (x) D2 (x) D3) C`` for every rotation, with the D
matrices of :mod:`maloq_b200.core.sph`.  It is built the way e3nn defines its ``wigner_3j``
(the convention of the reference's labels): the complex Clebsch-Gordan coefficients
<l1 m1 l2 m2 | l3 m3> (Racah's formula), carried into the real harmonic basis by the
change-of-basis matrices Q_l (with the (-i)^l factor that makes the result real),
``C = einsum(Q1, Q2, conj(Q3)^T, CG)``, divided by its Frobenius norm - in float64.  This fixes
the sign of every triple (the invariant subspace of l1 (x) l2 (x) l3 is one-dimensional, so
the tensors differ from any other construction by at most a sign).

The coupled<->uncoupled transform follows the reference's ``e3TensorDecomp``
(``fock_utils/utils_tensor_decomp.py:51-169``): an orbital block ``H[l1, l2]`` of shape
``(2l1+1) x (2l2+1)`` maps to coefficients ``c_l3 = (2 l3 + 1) sum_ij C(l3, l1, l2)_{k,i,j} H_ij``
(``get_net_out``) and back by ``H_ij = sum_k C(l1, l2, l3)_{i,j,k} c_k`` (``get_H``).
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch


def _clebsch_gordan(j1: int, m1: int, j2: int, m2: int, J: int, M: int) -> float:
    """<j1 m1 j2 m2 | J M> by Racah's formula (Condon-Shortley phases)."""
    if M != m1 + m2 or not abs(j1 - j2) <= J <= j1 + j2 or abs(m1) > j1 or abs(m2) > j2 or abs(M) > J:
        return 0.0
    f = math.factorial
    pre = math.sqrt((2 * J + 1) * f(J + j1 - j2) * f(J - j1 + j2) * f(j1 + j2 - J) / f(j1 + j2 + J + 1))
    pre *= math.sqrt(f(J + M) * f(J - M) * f(j1 - m1) * f(j1 + m1) * f(j2 - m2) * f(j2 + m2))
    s = 0.0
    for k in range(j1 + j2 - J + 1):
        a = (k, j1 + j2 - J - k, j1 - m1 - k, j2 + m2 - k, J - j2 + m1 + k, J - j1 - m2 + k)
        if min(a) < 0:
            continue
        s += (-1) ** k / math.prod(f(x) for x in a)
    return pre * s


def _real_to_complex(l: int) -> np.ndarray:
    """Q_l with (complex harmonic index, real harmonic index): real harmonics m < 0 / m > 0
    are the (sin, cos) combinations of the complex pair +-|m|, times (-i)^l so that the real
    3j tensors below are real."""
    q = np.zeros((2 * l + 1, 2 * l + 1), dtype=np.complex128)
    r = 1 / math.sqrt(2)
    for m in range(-l, 0):
        q[l + m, l + abs(m)] = r
        q[l + m, l - abs(m)] = -1j * r
    q[l, l] = 1.0
    for m in range(1, l + 1):
        q[l + m, l + m] = (-1) ** m * r
        q[l + m, l - m] = 1j * (-1) ** m * r
    return (-1j) ** l * q


@lru_cache(maxsize=None)
def _wigner_3j_np(l1: int, l2: int, l3: int) -> np.ndarray:
    if not (abs(l1 - l2) <= l3 <= l1 + l2):
        raise ValueError(f"l3={l3} not in |l1-l2|..l1+l2 for l1={l1}, l2={l2}")
    C = np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1))
    for m1 in range(-l1, l1 + 1):
        for m2 in range(-l2, l2 + 1):
            if abs(m1 + m2) <= l3:
                C[l1 + m1, l2 + m2, l3 + m1 + m2] = _clebsch_gordan(l1, m1, l2, m2, l3, m1 + m2)
    Cr = np.einsum("ij,kl,mn,ikn->jlm", _real_to_complex(l1), _real_to_complex(l2),
                   np.conj(_real_to_complex(l3).T), C.astype(np.complex128))
    assert np.abs(Cr.imag).max() < 1e-10
    Cr = Cr.real
    Cr = Cr / np.linalg.norm(Cr)
    Cr[np.abs(Cr) < 1e-14] = 0.0
    return np.ascontiguousarray(Cr)


def wigner_3j(l1: int, l2: int, l3: int, dtype=torch.float32, device=None) -> torch.Tensor:
    return torch.tensor(_wigner_3j_np(l1, l2, l3), dtype=dtype, device=device)


def l1l2_to_l3s(l1: int, l2: int) -> list[int]:
    """Coupled degrees for an l1 x l2 orbital block (diffuse shells are tagged l + 10)."""
    l1, l2 = l1 % 10, l2 % 10
    return list(range(abs(l1 - l2), l1 + l2 + 1))


class BasisTransform:
    """Dense block-diagonal coupled<->uncoupled transform for a list of (l1, l2) blocks.

    ``W`` [D, D]: coupled label row -> uncoupled block row (``get_H``);
    ``W_inv`` [D, D]: the inverse (``get_net_out``).  ``blocks`` lists, per orbital block,
    ``(l1, l2, coupled_start, uncoupled_start)`` for kernels that exploit the block
    structure instead of the dense matrix.
    Reference: ``fock_utils/utils_tensor_decomp.py:51-169``.
    """

    def __init__(self, out_js_list, dtype=torch.float32, device="cpu"):
        self.out_js_list = [(int(a), int(b)) for a, b in out_js_list]
        in_slices, h_slices = [0], [0]
        blocks = []
        wms, wms_H = [], []
        for l1, l2 in self.out_js_list:
            a, b = l1 % 10, l2 % 10
            l3s = l1l2_to_l3s(a, b)
            wm = np.concatenate([_wigner_3j_np(a, b, l3) for l3 in l3s], axis=-1)  # [d1, d2, sum d3]
            wmH = np.concatenate([_wigner_3j_np(l3, a, b) * (2 * l3 + 1) for l3 in l3s], axis=0)  # [sum d3, d1, d2]
            blocks.append((a, b, in_slices[-1], h_slices[-1]))
            in_slices.append(in_slices[-1] + sum(2 * l + 1 for l in l3s))
            h_slices.append(h_slices[-1] + (2 * a + 1) * (2 * b + 1))
            wms.append(wm)
            wms_H.append(wmH)
        self.in_slices, self.H_slices, self.blocks = in_slices, h_slices, blocks
        D_in, D_h = in_slices[-1], h_slices[-1]
        W = np.zeros((D_in, D_h))
        W_inv = np.zeros((D_h, D_in))
        for i in range(len(self.out_js_list)):
            i0, i1, h0, h1 = in_slices[i], in_slices[i + 1], h_slices[i], h_slices[i + 1]
            W[i0:i1, h0:h1] = wms[i].reshape(h1 - h0, i1 - i0).T
            W_inv[h0:h1, i0:i1] = wms_H[i].reshape(i1 - i0, h1 - h0).T
        self.W_global = torch.tensor(W, dtype=dtype, device=device)
        self.W_global_inv = torch.tensor(W_inv, dtype=dtype, device=device)
        self.dim = D_in

    def to(self, device=None, dtype=None):
        self.W_global = self.W_global.to(device=device, dtype=dtype)
        self.W_global_inv = self.W_global_inv.to(device=device, dtype=dtype)
        return self

    def column_tables(self, inverse: bool, transpose: bool = False):
        """Per output column u of the transform (``inverse`` = uncoupled -> coupled;
        ``transpose`` = multiply by the transposed matrix, the backward of the transform):
        ``meta[u] = (s, n, c, 0)`` and ``coef`` such that
        ``out[:, u] = sum_{j<n} in[:, s + j] * coef[c + j * n]`` (one square CG block per orbital
        shell pair; coefficients of adjacent columns of a block are adjacent)."""
        key = f"_tables_{'inv' if inverse else 'fwd'}{'_t' if transpose else ''}"
        if getattr(self, key, None) is None:
            W = (self.W_global_inv if inverse else self.W_global).detach().cpu().double().numpy()
            src = self.H_slices if inverse else self.in_slices
            dst = self.in_slices if inverse else self.H_slices
            if transpose:
                W, src, dst = W.T, dst, src
            meta = np.zeros((self.dim, 4), dtype=np.int32)
            coef = []
            base = 0
            for g in range(len(self.out_js_list)):
                s0, s1, d0, d1 = src[g], src[g + 1], dst[g], dst[g + 1]
                n = s1 - s0
                blk = W[s0:s1, d0:d1]  # [j, k]
                coef.append(blk.reshape(-1))
                for k in range(n):
                    meta[d0 + k] = (s0, n, base + k, 0)
                base += n * n
            setattr(self, key, (meta, np.concatenate(coef)))
        return getattr(self, key)

    def get_H(self, net_out: torch.Tensor) -> torch.Tensor:
        from ..ops import basis_transform as bt

        return bt.apply_transform(net_out, self, inverse=False)

    def get_net_out(self, H: torch.Tensor) -> torch.Tensor:
        from ..ops import basis_transform as bt

        return bt.apply_transform(H, self, inverse=True)
