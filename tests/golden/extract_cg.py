"""Extract the e3nn 0.4.4 real-basis coupling constants the reference ships
(mace/src/cg.inc) into tests/golden/cg_e3nn044.txt, one "l1 l2 lo a b c value" row per
line.  Run once where the reference tree is available:

    python tests/golden/extract_cg.py <reference tree>/mace/src/cg.inc
"""
import re
import sys
from pathlib import Path

rows = []
for line in Path(sys.argv[1]).read_text().splitlines():
    m = re.match(r"\s*\{([^}]*)\},", line)
    if m:
        rows.append(" ".join(x.strip() for x in m.group(1).split(",")))
Path(__file__).with_name("cg_e3nn044.txt").write_text("\n".join(rows) + "\n")
