"""Orbital basis sets: shell angular momenta per element (Z -> list of l).

The def2-SVP tables list the standard def2-SVP shell structure of each element (a
chemistry fact, identical to the reference's ``fock_utils/basis_sets.py:3-26``).  The
synthetic sets size the benchmark configurations:

* ``split_valence_small``: H 2s1p (5 orbitals), C/N/O 3s2p1d (14);
* ``def2_svp_like``: H 5, second-row 14, S/Cl 18 orbitals;
* ``def2_tzvp_like``: 6-31 orbitals per element with shells up to f (lmax of labels 6);
* ``dzvp_like``: 13 orbitals per Si and O (2s2p1d), 25 for Hf (6s3p2d).
"""

H, C, N, O, F, P, S, Cl, Br, Si, Hf = 1, 6, 7, 8, 9, 15, 16, 17, 35, 14, 72

orbital_basis_def2_svp_nabla = {35: [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2], 17: [0, 0, 0, 0, 1, 1, 1, 2],
                                16: [0, 0, 0, 0, 1, 1, 1, 2], 9: [0, 0, 0, 1, 1, 2], 8: [0, 0, 0, 1, 1, 2],
                                7: [0, 0, 0, 1, 1, 2], 6: [0, 0, 0, 1, 1, 2], 1: [0, 0, 1]}

orbital_basis_def2_svp_QM7 = {9: [0, 0, 0, 1, 1, 2], 8: [0, 0, 0, 1, 1, 2], 7: [0, 0, 0, 1, 1, 2],
                              6: [0, 0, 0, 1, 1, 2], 1: [0, 0, 1]}

split_valence_small = {H: [0, 0, 1], C: [0, 0, 0, 1, 1, 2], N: [0, 0, 0, 1, 1, 2], O: [0, 0, 0, 1, 1, 2]}

def2_svp_like = {H: [0, 0, 1], C: [0, 0, 0, 1, 1, 2], N: [0, 0, 0, 1, 1, 2], O: [0, 0, 0, 1, 1, 2],
                 F: [0, 0, 0, 1, 1, 2], S: [0, 0, 0, 0, 1, 1, 1, 2], Cl: [0, 0, 0, 0, 1, 1, 1, 2]}

# 6..31 orbitals, shells up to f
def2_tzvp_like = {H: [0, 0, 0, 1],                                   # 6
                  C: [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3],               # 31
                  N: [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3],               # 31
                  O: [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3],               # 31
                  F: [0, 0, 0, 0, 0, 1, 1, 1, 2, 2, 3],               # 31
                  P: [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 3],               # 29
                  S: [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 3],               # 29
                  Cl: [0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 3],              # 29
                  Br: [0, 0, 0, 0, 1, 1, 1, 2, 2, 3]}                 # 30

# Si/O 2s2p1d = 13 orbitals; Hf 6s3p2d = 25 orbitals (label lmax 4)
dzvp_like = {Si: [0, 0, 1, 1, 2], O: [0, 0, 1, 1, 2], Hf: [0, 0, 0, 0, 0, 0, 1, 1, 1, 2, 2]}


def n_orbitals(basis: dict, z: int) -> int:
    return sum(2 * l + 1 for l in basis[z])


BASIS_SETS = {
    "def2_svp_nabla": orbital_basis_def2_svp_nabla,
    "def2_svp_qm7": orbital_basis_def2_svp_QM7,
    "split_valence_small": split_valence_small,
    "def2_svp_like": def2_svp_like,
    "def2_tzvp_like": def2_tzvp_like,
    "dzvp_like": dzvp_like,
}


def get_basis(name_or_dict):
    if isinstance(name_or_dict, dict):
        return {int(k): list(v) for k, v in name_or_dict.items()}
    return {int(k): list(v) for k, v in BASIS_SETS[name_or_dict].items()}
