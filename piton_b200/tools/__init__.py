"""Command-line tools of the B200 backend (``python -m piton_b200.tools.compile``)."""
