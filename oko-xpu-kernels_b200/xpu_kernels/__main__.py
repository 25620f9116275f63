"""``python -m xpu_kernels`` -- self-test the INT8 library on this machine."""

from __future__ import annotations

import sys

from . import int8


def main() -> int:
    return 0 if int8.selftest() else 1


if __name__ == "__main__":
    sys.exit(main())
