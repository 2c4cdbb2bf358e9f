"""Operator modules with the reference's names and signatures."""
