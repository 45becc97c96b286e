"""Model-side callers of the decode path."""
