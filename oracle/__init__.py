"""Parity oracle for the triangle hot path (test infrastructure; never imported by the product)."""
