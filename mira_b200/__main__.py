"""`python -m mira_b200 run prog.mira -t cuda --quantize w8a8 [--check]`: MIRA's own CLI
(mira/cli.py) with the cuda target registered."""
import sys

from .plugin import install


def main(argv=None) -> int:
    install()
    from mira.cli import main as mira_main
    return mira_main(argv)


if __name__ == "__main__":
    sys.exit(main())
