"""Command-line entry points: ``python -m predicitivecoding_b200.cli.translate``,
``python -m predicitivecoding_b200.cli.demos`` and ``python -m predicitivecoding_b200.cli.mixed_precision_bench``."""
