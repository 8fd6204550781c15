"""Command-line entry points mirroring the reference's run/ scripts that sit on the hot path."""
