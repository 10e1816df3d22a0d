"""Offline analysis of trained models (embedding projections and clustering)."""
