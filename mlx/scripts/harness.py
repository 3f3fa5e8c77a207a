#!/usr/bin/env python3
"""Entry point kept at the reference's path (mlx/scripts/harness.py); the
harness itself is metalbench_b200.harness."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from metalbench_b200.harness import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())
