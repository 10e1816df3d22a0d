"""Real spherical harmonics, Wigner-D matrices and J matrices (y-up convention).

Convention (the one used by the reference's e3nn-based model, ``helm/common/rotation.py:68-83``
and ``helm/esen_osh.py:316-318``): the polar axis is ``y``; the azimuth is
``phi = atan2(x, z)``; inside a degree ``l`` the components are ordered ``m = -l..l``;
``m > 0`` is the cosine-like component, ``m < 0`` the sine-like one; no Condon-Shortley
phase.  With this convention the degree-1 harmonics are proportional to ``(x, y, z)``.

Everything here is built from the mathematics stated in the docstrings:

* harmonics: associated Legendre functions by the standard upward recurrence, times
  ``cos(m phi)`` / ``sin(|m| phi)``;
* the D matrix of a 3x3 matrix ``R`` in this basis: the unique linear map with
  ``Y_l(R r) = D_l(R) Y_l(r)`` for all unit vectors ``r``, found by least squares on a
  fixed point set (exact up to rounding because degree-``l`` harmonics span a
  ``2l+1``-dimensional space closed under rotation);
* ``J_l = D_l(P)`` with ``P`` the x<->-y swap, so that a rotation about ``x`` is
  ``J X(beta) J`` with ``X`` the rotation about the polar axis;
* ``D(alpha, beta, gamma) = X(alpha) J X(beta) J X(gamma)`` for Euler angles of
  ``R = R_y(alpha) R_x(beta) R_y(gamma)`` (the ZYZ-style formula of e3nn 0.4, written
  for a y polar axis).

The J matrices are stored in backbone checkpoints as the buffers ``Jd_{l}``
(reference ``helm/esen_osh.py:125-127``), so they are generated here bit-for-bit in the
same convention.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch

# The reflection that maps x -> -y, y -> -x, z -> z.  It conjugates a rotation about the
# polar (y) axis into a rotation about x (up to the sign of the angle).
_P_SWAP = np.array([[0.0, -1.0, 0.0], [-1.0, 0.0, 0.0], [0.0, 0.0, 1.0]])


def _assoc_legendre(lmax: int, t: np.ndarray) -> dict:
    """P_l^m(t) for 0 <= m <= l <= lmax without the Condon-Shortley phase.

    Uses P_m^m = (2m-1)!! (1-t^2)^{m/2}, P_{m+1}^m = (2m+1) t P_m^m and
    (l-m) P_l^m = (2l-1) t P_{l-1}^m - (l+m-1) P_{l-2}^m.
    """
    s = np.sqrt(np.clip(1.0 - t * t, 0.0, None))
    P = {}
    pmm = np.ones_like(t)
    for m in range(lmax + 1):
        if m > 0:
            pmm = pmm * (2 * m - 1) * s
        P[(m, m)] = pmm
        if m + 1 <= lmax:
            P[(m + 1, m)] = (2 * m + 1) * t * pmm
        for l in range(m + 2, lmax + 1):
            P[(l, m)] = ((2 * l - 1) * t * P[(l - 1, m)] - (l + m - 1) * P[(l - 2, m)]) / (l - m)
    return P


def real_sph_harm(l: int, xyz: np.ndarray) -> np.ndarray:
    """Real spherical harmonics of degree ``l`` at unit vectors ``xyz`` [n, 3] -> [n, 2l+1].

    "Component" normalisation: the mean of Y_lm^2 over the sphere is 1 for every m.
    """
    xyz = np.asarray(xyz, dtype=np.float64)
    x, y, z = xyz[:, 0], xyz[:, 1], xyz[:, 2]
    t = np.clip(y, -1.0, 1.0)
    phi = np.arctan2(x, z)
    P = _assoc_legendre(l, t)
    out = np.zeros((xyz.shape[0], 2 * l + 1))
    for m in range(-l, l + 1):
        am = abs(m)
        # component normalisation: sqrt((2l+1) (l-|m|)!/(l+|m|)! * (2 - delta_m0))
        n = math.sqrt((2 * l + 1) * math.factorial(l - am) / math.factorial(l + am) * (1 if m == 0 else 2))
        if m > 0:
            ang = np.cos(am * phi)
        elif m < 0:
            ang = np.sin(am * phi)
        else:
            ang = np.ones_like(phi)
        out[:, m + l] = n * P[(l, am)] * ang
    return out


@lru_cache(maxsize=None)
def _fit_points(l: int) -> np.ndarray:
    rng = np.random.default_rng(1234 + l)
    v = rng.normal(size=(8 * (2 * l + 1) + 16, 3))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def wigner_D_from_matrix(l: int, R: np.ndarray) -> np.ndarray:
    """D_l(R) with Y_l(R r) = D_l(R) Y_l(r) (least-squares on a fixed point set)."""
    r = _fit_points(l)
    Y = real_sph_harm(l, r)  # [n, d]
    YR = real_sph_harm(l, r @ np.asarray(R, dtype=np.float64).T)  # [n, d]
    # YR^T = D Y^T  ->  D = YR^T pinv(Y^T)
    D = np.linalg.lstsq(Y, YR, rcond=None)[0].T
    return D


@lru_cache(maxsize=None)
def J_matrix(l: int) -> np.ndarray:
    """J_l = D_l(P) for the x <-> -y reflection P; entries rounded to remove fit noise."""
    J = wigner_D_from_matrix(l, _P_SWAP)
    J[np.abs(J) < 1e-12] = 0.0
    return J


def J_matrices(lmax: int, dtype=torch.float64) -> list[torch.Tensor]:
    return [torch.tensor(J_matrix(l), dtype=dtype) for l in range(lmax + 1)]


def polar_rot_mat(angle: torch.Tensor, l: int) -> torch.Tensor:
    """X_l(angle): rotation about the polar axis in the degree-l block, [..., 2l+1, 2l+1].

    Row i (m = i - l) has cos(f angle) on the diagonal and sin(f angle) at column 2l - i,
    with f = l - i.
    """
    M = angle.new_zeros((*angle.shape, 2 * l + 1, 2 * l + 1))
    for i in range(2 * l + 1):
        f = l - i
        M[..., i, 2 * l - i] = torch.sin(f * angle)
        M[..., i, i] = torch.cos(f * angle)
    return M


def wigner_D(l: int, alpha: torch.Tensor, beta: torch.Tensor, gamma: torch.Tensor, J: torch.Tensor) -> torch.Tensor:
    """D_l(alpha, beta, gamma) = X(alpha) J X(beta) J X(gamma)."""
    alpha, beta, gamma = torch.broadcast_tensors(alpha, beta, gamma)
    J = J.to(alpha.dtype)
    return polar_rot_mat(alpha, l) @ J @ polar_rot_mat(beta, l) @ J @ polar_rot_mat(gamma, l)


def euler_matrix(alpha, beta, gamma) -> np.ndarray:
    """R = R_y(alpha) R_x(beta) R_y(gamma) (right-handed, active rotations)."""

    def ry(a):
        c, s = math.cos(a), math.sin(a)
        return np.array([[c, 0, s], [0, 1, 0], [-s, 0, c]])

    def rx(a):
        c, s = math.cos(a), math.sin(a)
        return np.array([[1, 0, 0], [0, c, -s], [0, s, c]])

    return ry(alpha) @ rx(beta) @ ry(gamma)


def edge_euler_angles(vec_yzx: torch.Tensor):
    """(alpha, beta) of unit vectors given in the model frame (x, y, z) = (y_in, z_in, x_in).

    beta = acos(y) is the polar angle from the y axis and alpha = atan2(x, z) the azimuth;
    the rotation R_y(alpha) R_x(beta) maps the polar axis onto the vector.
    Reference: ``helm/common/rotation.py:86-99``.
    """
    v = torch.nn.functional.normalize(vec_yzx, dim=-1).clamp(-1.0, 1.0)
    x, y, z = v.unbind(-1)
    beta = torch.acos(y)
    alpha = torch.atan2(x, z)
    return alpha, beta


def block_diag_wigner(lmax: int, alpha, beta, gamma, Js) -> torch.Tensor:
    """Block-diagonal [(L+1)^2, (L+1)^2] D(alpha, beta, gamma) per batch element."""
    size = (lmax + 1) ** 2
    out = alpha.new_zeros((*alpha.shape, size, size))
    s = 0
    for l in range(lmax + 1):
        d = 2 * l + 1
        out[..., s : s + d, s : s + d] = wigner_D(l, alpha, beta, gamma, Js[l])
        s += d
    return out


def rotation_to_wigner_numeric(lmax: int, R: np.ndarray) -> np.ndarray:
    """Block-diagonal D(R) (numeric fit), used by tests to rotate features."""
    size = (lmax + 1) ** 2
    out = np.zeros((size, size))
    s = 0
    for l in range(lmax + 1):
        d = 2 * l + 1
        out[s : s + d, s : s + d] = wigner_D_from_matrix(l, R)
        s += d
    return out
