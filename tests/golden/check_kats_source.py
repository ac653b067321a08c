"""Re-reads the known-answer vectors of reference_kats.json from the
reference's own test source, to show where each number came from.

Run where ynishi/beatlm is mounted (``python tests/golden/check_kats_source.py
/path/to/beatlm``); it prints each vector's source range and fails if a
transcribed literal does not occur there. The GPU box has no reference, so the
test suite never runs this; it only reads the JSON.
"""
import json
import os
import re
import sys


def literals(text):
    """Every numeric literal of a Rust source range, underscores removed."""
    return {float(m.replace("_", "")) for m in re.findall(r"-?\d[\d_]*\.?[\d_]*(?:e-?\d+)?", text)}


def main(root):
    kats = json.load(open(os.path.join(os.path.dirname(__file__), "reference_kats.json")))
    bad = 0
    for name, entry in kats.items():
        if name.startswith("_") or "source" not in entry:
            continue
        m = re.match(r"([\w/.-]+):(\d+)-(\d+)", entry["source"])
        path, lo, hi = m.group(1), int(m.group(2)), int(m.group(3))
        lines = open(os.path.join(root, path)).read().splitlines()[lo - 1:hi]
        found = literals("\n".join(lines))
        wanted = []
        for key, val in entry.items():
            if isinstance(val, list) and all(isinstance(v, (int, float)) for v in val):
                wanted += [abs(float(v)) for v in val]
        missing = sorted({v for v in wanted if v not in {abs(f) for f in found}})
        status = "ok" if not missing else "MISSING %s" % missing[:8]
        bad += bool(missing)
        print("%-20s %-55s %s" % (name, entry["source"], status))
    return 1 if bad else 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python check_kats_source.py /path/to/beatlm (the reference's root)")
    sys.exit(main(sys.argv[1]))
