"""Attention ops and the paged dense runner (drop-in for plastic_infer.exec)."""
