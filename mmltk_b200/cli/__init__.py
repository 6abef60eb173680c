"""Command line (``mmltk``)."""
from .main import build_parser, main, train_options_from_args

__all__ = ["build_parser", "main", "train_options_from_args"]
