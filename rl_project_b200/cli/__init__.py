"""Command-line interface (``forgeline-b200`` / ``python -m rl_project_b200.cli``)."""

from rl_project_b200.cli.main import build_parser, main

__all__ = ["build_parser", "main"]
