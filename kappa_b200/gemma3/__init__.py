"""Gemma3 W8 MLP with kappa's signature (kappa/gemma3/ffn.py)."""
