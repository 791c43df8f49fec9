"""Qwen3 W8 FFN / MoE functions with kappa's signatures (kappa/qwen3/)."""
