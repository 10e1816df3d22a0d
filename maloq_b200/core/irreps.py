"""Irreducible-representation bookkeeping (all irreps are even parity, as in the reference).

A small, self-contained replacement for the parts of ``e3nn.o3.Irreps`` the reference uses
(``helm/common/irreps_utils.py``, ``fock_utils/utils_tensor_decomp.py:206-306``):

* :class:`Irreps` - an ordered list of ``(mul, l)`` with ``dim``, ``ls``, ``count``,
  ``sort`` and ``simplify``; string form ``"64x0e+64x1e"``;
* product irreps of an ``l1 x l2`` orbital block;
* the orbital-shell list (``ls_list``) of a basis set and the label layout of every
  shell pair;
* node-block symmetry reductions (``reduce_node`` / ``reduce_node_intra``) and the
  half-edge (alpha/beta) reduction used by the Fock head.
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class _MulIr:
    mul: int
    l: int

    @property
    def dim(self) -> int:
        return self.mul * (2 * self.l + 1)


class Irreps:
    """Ordered direct sum of ``mul x l`` (even parity) irreps."""

    def __init__(self, spec=None):
        items: list[_MulIr] = []
        if spec is None or spec == "":
            pass
        elif isinstance(spec, Irreps):
            items = list(spec._items)
        elif isinstance(spec, str):
            for tok in spec.split("+"):
                tok = tok.strip()
                if not tok:
                    continue
                m = re.fullmatch(r"(?:(\d+)x)?(\d+)([eo]?)", tok)
                if m is None:
                    raise ValueError(f"bad irreps token {tok!r}")
                items.append(_MulIr(int(m.group(1) or 1), int(m.group(2))))
        else:
            for it in spec:
                if isinstance(it, _MulIr):
                    items.append(it)
                else:
                    mul, ir = it
                    l = ir[0] if isinstance(ir, (tuple, list)) else int(ir)
                    items.append(_MulIr(int(mul), int(l)))
        self._items = tuple(items)

    def __iter__(self):
        return iter(self._items)

    def __len__(self):
        return len(self._items)

    def __getitem__(self, i):
        return self._items[i]

    def __add__(self, other):
        return Irreps(list(self._items) + list(Irreps(other)._items))

    def __eq__(self, other):
        return isinstance(other, Irreps) and self._items == other._items

    def __hash__(self):
        return hash(self._items)

    def __repr__(self):
        return "+".join(f"{it.mul}x{it.l}e" for it in self._items)

    __str__ = __repr__

    @property
    def dim(self) -> int:
        return sum(it.dim for it in self._items)

    @property
    def num_irreps(self) -> int:
        return sum(it.mul for it in self._items)

    @property
    def ls(self) -> list[int]:
        return [it.l for it in self._items for _ in range(it.mul)]

    @property
    def lmax(self) -> int:
        return max(it.l for it in self._items)

    def count(self, l) -> int:
        if isinstance(l, str):
            l = int(l.rstrip("eo"))
        return sum(it.mul for it in self._items if it.l == l)

    def sort(self):
        """(sorted irreps, p, inv): sorted[i] = self[inv[i]], self[i] = sorted[p[i]] (stable by l)."""
        inv = sorted(range(len(self._items)), key=lambda i: (self._items[i].l, i))
        p = [0] * len(inv)
        for new, old in enumerate(inv):
            p[old] = new
        return Irreps([self._items[i] for i in inv]), p, inv

    def simplify(self):
        out: list[_MulIr] = []
        for it in self._items:
            if out and out[-1].l == it.l:
                out[-1] = _MulIr(out[-1].mul + it.mul, it.l)
            elif it.mul > 0:
                out.append(it)
        return Irreps(out)

    def slices(self):
        s, out = 0, []
        for it in self._items:
            out.append((s, s + it.dim))
            s += it.dim
        return out


def product_ls(l1: int, l2: int, kind: str = "all") -> list[int]:
    l3s = range(abs(l1 - l2), l1 + l2 + 1)
    if kind == "even":
        return [l for l in l3s if l % 2 == 0]
    if kind == "odd":
        return [l for l in l3s if l % 2 == 1]
    return list(l3s)


def product_irreps(l1: int, l2: int, kind: str | None = None) -> Irreps:
    return Irreps([(1, l) for l in product_ls(l1 % 10, l2 % 10, kind or "all")])


# ---------------------------------------------------------------------------------------
# orbital bases -> label layout
# ---------------------------------------------------------------------------------------

def tag_diffuse(orbitals: list[int]) -> list[int]:
    """Shells after the first decrease of l are diffuse; they are tagged l + 10."""
    start = len(orbitals)
    for i in range(1, len(orbitals)):
        if orbitals[i] < orbitals[i - 1]:
            start = i
            break
    return [l if i < start else l + 10 for i, l in enumerate(orbitals)]


@dataclass
class LabelLayout:
    """Label layout of an orbital basis.

    ``ls_list``: shell slots (diffuse tagged +10), e.g. [0,0,0,1,1,2];
    ``out_js_list``: (l1, l2) of every slot pair, row-major;
    ``slot_offsets``: start of each slot pair's block in a label row (len n^2 + 1);
    ``irreps_out``: product irreps of all slot pairs (coupled basis, same offsets);
    ``template``: {(Zi, Zj): [(r0, r1, c0, c1, out0), ...]} mapping an atom-pair Fock
    block's sub-block to its label slice;
    ``orbitals_per_element``: {Z: number of orbitals}.
    Reference: ``fock_utils/utils_tensor_decomp.py:206-373`` and
    ``fock_utils/matrix2labels_kernels.py:1232-1271``.
    """

    ls_list: list[int]
    out_js_list: list[tuple[int, int]]
    slot_offsets: list[int]
    irreps_out: Irreps
    template: dict
    orbitals_per_element: dict
    shell_offsets: dict

    @property
    def target_len(self) -> int:
        return self.slot_offsets[-1]

    @property
    def lmax(self) -> int:
        return self.irreps_out.lmax


def make_label_layout(orbital_basis: dict) -> LabelLayout:
    tagged = {int(Z): tag_diffuse(list(orbs)) for Z, orbs in orbital_basis.items()}
    ls_list: list[int] = []
    for l in range(20):
        ls_list += [l] * max(sum(1 for o in orbs if o == l) for orbs in tagged.values())
    n = len(ls_list)
    out_js = [(ls_list[p], ls_list[q]) for p in range(n) for q in range(n)]
    offsets = [0]
    irreps = Irreps()
    for l1, l2 in out_js:
        pi = product_irreps(l1, l2)
        irreps = irreps + pi
        offsets.append(offsets[-1] + pi.dim)

    # slot of the k-th shell of an element: the k'-th slot with the same tagged l, where k'
    # counts earlier shells of the element with that tagged l
    def slots_of(orbs):
        out = []
        for k, l in enumerate(orbs):
            rank = sum(1 for j in range(k) if orbs[j] == l)
            cand = [s for s, ls in enumerate(ls_list) if ls == l]
            out.append(cand[rank])
        return out

    shell_offsets = {}
    for Z, orbs in tagged.items():
        starts = np.concatenate([[0], np.cumsum([2 * (l % 10) + 1 for l in orbs])]).astype(int)
        shell_offsets[Z] = starts.tolist()
    template = {}
    for Zi, oi in tagged.items():
        si = slots_of(oi)
        for Zj, oj in tagged.items():
            sj = slots_of(oj)
            entries = []
            for a, la in enumerate(oi):
                for b, lb in enumerate(oj):
                    slot = si[a] * n + sj[b]
                    entries.append((shell_offsets[Zi][a], shell_offsets[Zi][a + 1],
                                    shell_offsets[Zj][b], shell_offsets[Zj][b + 1], offsets[slot]))
            entries.sort(key=lambda e: e[4])
            template[(Zi, Zj)] = entries
    norb = {Z: shell_offsets[Z][-1] for Z in tagged}
    return LabelLayout(ls_list, out_js, offsets, irreps, template, norb, shell_offsets)


def layout_masks(layout: LabelLayout, max_z: int = 100):
    """Boolean label masks per element pair: mask[(Zi, Zj)] -> bool[target_len]."""
    out = {}
    for key, entries in layout.template.items():
        m = np.zeros(layout.target_len, dtype=bool)
        for r0, r1, c0, c1, o in entries:
            m[o : o + (r1 - r0) * (c1 - c0)] = True
        out[key] = m
    return out


# ---------------------------------------------------------------------------------------
# head symmetry reductions (reference helm/common/irreps_utils.py:10-221)
# ---------------------------------------------------------------------------------------

def _ls(ls_list):
    return [l % 10 for l in ls_list]


def all_indices_dict(ls_list):
    ls_list = _ls(ls_list)
    d, idx = {}, 0
    for i, li in enumerate(ls_list):
        for j, lj in enumerate(ls_list):
            for l in product_ls(li, lj):
                d[(i, j, l)] = idx
                idx += 2 * l + 1
    return d


def reduced_indices_dict(ls_list, reduce_node_intra=False):
    ls_list = _ls(ls_list)
    d, idx = {}, 0
    kind = "even" if reduce_node_intra else "all"
    for i, li in enumerate(ls_list):
        for j, lj in enumerate(ls_list):
            if i == j:
                prod = product_ls(li, lj, kind)
            elif i < j:
                prod = product_ls(li, lj)
            else:
                continue
            for l in prod:
                d[(i, j, l)] = idx
                idx += 2 * l + 1
    return d


def reduced_node_irreps(ls_list, reduce_node_intra=False) -> Irreps:
    ls_list = _ls(ls_list)
    kind = "even" if reduce_node_intra else "all"
    items = []
    for i, li in enumerate(ls_list):
        for j, lj in enumerate(ls_list):
            if i == j:
                items += [(1, l) for l in product_ls(li, lj, kind)]
            elif i < j:
                items += [(1, l) for l in product_ls(li, lj)]
    return Irreps(items)


def reduced_to_all_indices(ls_list, reduce_node_intra=False) -> list[int]:
    """Gather index (reduced -> full label); -1 marks removed odd self-interaction irreps."""
    ls_list = _ls(ls_list)
    red = reduced_indices_dict(ls_list, reduce_node_intra)
    out = []
    for i, li in enumerate(ls_list):
        for j, lj in enumerate(ls_list):
            for l in product_ls(li, lj):
                n = 2 * l + 1
                if (i, j, l) in red:
                    s = red[(i, j, l)]
                elif i == j:
                    assert reduce_node_intra
                    out += [-1] * n
                    continue
                else:
                    s = red[(j, i, l)]
                out += list(range(s, s + n))
    return out


def parity_multiplier(ls_list, reduce_node_intra=False) -> list[float]:
    """+1/-1/0 per full label entry: lower-triangle blocks pick up (-1)^(l1+l2+l3)."""
    ls_list = _ls(ls_list)
    full = all_indices_dict(ls_list)
    total = sum(2 * l + 1 for (_, _, l) in full)
    mult = [1.0] * total
    for i, li in enumerate(ls_list):
        for j, lj in enumerate(ls_list):
            if i == j and reduce_node_intra:
                for l in product_ls(li, lj, "odd"):
                    s = full[(i, j, l)]
                    mult[s : s + 2 * l + 1] = [0.0] * (2 * l + 1)
            elif i > j:
                kind = "even" if (li + lj) % 2 == 1 else "odd"
                for l in product_ls(li, lj, kind):
                    s = full[(i, j, l)]
                    mult[s : s + 2 * l + 1] = [-1.0] * (2 * l + 1)
    return mult


def sorted_to_original_permutation(irreps: Irreps) -> list[int]:
    """Index list ``perm`` with ``original = sorted_by_l[:, perm]``.

    The head produces its outputs grouped by l (sorted, stable); this permutation restores
    the label order.  Reference: ``helm/esen_osh.py:838-880``.
    """
    sorted_irreps, p, _ = irreps.sort()
    sorted_starts = np.concatenate([[0], np.cumsum([it.dim for it in sorted_irreps])]).astype(int)
    perm = []
    for k, it in enumerate(irreps):
        s = sorted_starts[p[k]]
        perm += list(range(s, s + it.dim))
    return perm


def edge_reduced_irreps(ls_list):
    """Alpha (symmetric) / beta (antisymmetric) half-edge irreps and index bookkeeping.

    Returns (irreps_alpha, irreps_beta, parity_flip_indices, off_diag_alpha, off_diag_beta).
    Reference: ``helm/esen_osh.py:736-836``.
    """
    ls_list = _ls(ls_list)
    alpha, beta, flips = [], [], []
    ptr = 0
    for i, l1 in enumerate(ls_list):
        for j, l2 in enumerate(ls_list):
            prod = product_ls(l1, l2)
            if i == j:
                alpha += [(1, l) for l in product_ls(l1, l2, "even")]
                beta += [(1, l) for l in product_ls(l1, l2, "odd")]
                ptr += sum(2 * l + 1 for l in prod)
            elif i < j:
                alpha += [(1, l) for l in prod]
                par = (l1 + l2) % 2
                for l in prod:
                    if (par == 0 and l % 2 == 1) or (par == 1 and l % 2 == 0):
                        flips += list(range(ptr, ptr + 2 * l + 1))
                    ptr += 2 * l + 1
            else:
                beta += [(1, l) for l in prod]
                ptr += sum(2 * l + 1 for l in prod)
    a_blocks, b_blocks = {}, {}
    at = bt = 0
    for i, l1 in enumerate(ls_list):
        for j, l2 in enumerate(ls_list):
            prod = product_ls(l1, l2)
            dim = sum(2 * l + 1 for l in prod)
            if i == j:
                at += sum(2 * l + 1 for l in product_ls(l1, l2, "even"))
                bt += sum(2 * l + 1 for l in product_ls(l1, l2, "odd"))
            elif i < j:
                a_blocks[(i, j)] = np.arange(at, at + dim)
                at += dim
            else:
                b_blocks[(i, j)] = np.arange(bt, bt + dim)
                bt += dim
    offa = [v for (i, j), v in a_blocks.items()]
    offb = [b_blocks[(j, i)] for (i, j) in a_blocks]
    offa = np.concatenate(offa) if offa else np.zeros(0, dtype=np.int64)
    offb = np.concatenate(offb) if offb else np.zeros(0, dtype=np.int64)
    return Irreps(alpha), Irreps(beta), flips, offa, offb


def subspace_remix_permutation(irreps_alpha: Irreps, irreps_beta: Irreps, ls_list) -> list[int]:
    """Index list that interleaves [alpha | beta] outputs back into full label order."""
    ls_list = _ls(ls_list)

    def pool(irreps, start):
        out, cur = [], start
        for it in irreps:
            out.append(list(range(cur, cur + it.dim)))
            cur += it.dim
        return out

    pa, pb = pool(irreps_alpha, 0), pool(irreps_beta, irreps_alpha.dim)
    perm, ta, tb = [], 0, 0
    for i, l1 in enumerate(ls_list):
        for j, l2 in enumerate(ls_list):
            for l in product_ls(l1, l2):
                if i == j:
                    if l % 2 == 0:
                        perm += pa[ta]
                        ta += 1
                    else:
                        perm += pb[tb]
                        tb += 1
                elif i < j:
                    perm += pa[ta]
                    ta += 1
                else:
                    perm += pb[tb]
                    tb += 1
    return perm
