"""Append the GPU's packed section to a .l3m file (l3m_write_packed in include/l3m.h).

    python -m l3m_b200.pack model.l3m model-b200.l3m

The output is the input file unchanged plus every matrix the decode kernel streams, already in its
16-row tile order ("b200v1." tensors), and a new table of contents. The reference's reader (format
v1) accepts it and ignores the extra tensors; l3m_load copies them instead of repacking rows. No GPU
is needed.
"""
import sys


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__.strip().splitlines()[2].strip(), file=sys.stderr)
        return 2
    from . import lib
    return 0 if lib().l3m_write_packed(argv[0].encode(), argv[1].encode()) == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
