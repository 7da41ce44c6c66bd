"""Decoder architectures: logical tensor layout and initialisation."""
