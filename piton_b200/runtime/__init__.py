"""Launch path: binding (launcher.py) and the CUDA backend (cuda/)."""
