#!/usr/bin/env python3
"""Write tests/golden/codebook.json by running the reference's own codebook
generator (Jadon-Fox/glint glint_codec.py:87-113 _voronoi / build_cells and
glint_codec.py:162-172 write_c_header), imported from a read-only checkout given
by --ref (default: the GLINT_REFERENCE environment variable).

Recorded: the Voronoi bounds and the 256 children as exact f64 hex strings, and
the header text write_c_header produces.  The fixture is committed, so the tests
never need the reference at run time.
Run:  python tests/golden/make_codebook_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

OUT = Path(__file__).resolve().parent / "codebook.json"


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GLINT_REFERENCE", ""))
    args = ap.parse_args()
    if not args.ref or not Path(args.ref, "glint_codec.py").is_file():
        print("need --ref pointing at a Jadon-Fox/glint checkout", file=sys.stderr)
        return 2
    sys.path.insert(0, str(Path(args.ref).resolve()))
    import glint_codec  # noqa: E402

    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "glint_cells.h"
        glint_codec.write_c_header(str(p))
        header = p.read_text(encoding="utf-8")
    doc = {
        "source": "glint_codec.py (_voronoi, build_cells, write_c_header)",
        "voronoi_hex": [float(b).hex() for b in glint_codec._voronoi()],
        "cells_hex": [float(v).hex() for row in glint_codec.build_cells() for v in row],
        "header_text": header,
    }
    OUT.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
