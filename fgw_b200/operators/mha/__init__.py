"""Paged multi-head attention forward (FGW ``operators.mha``) for B200."""
