"""Electronic-structure evaluation of predicted Hamiltonians (orbitals, densities, energies)."""
