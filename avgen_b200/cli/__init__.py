"""The ``avgen-b200`` command line."""
from avgen_b200.cli.main import build_parser, main

__all__ = ["build_parser", "main"]
