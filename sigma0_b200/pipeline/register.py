"""Keep a generated markdown section in step with its JSON source.

The reference's ``tools/render_register.py`` renders a defect register kept as JSON into
the tables of a hand-written document, between two marker comments, and its ``--check``
mode fails when the document is stale (so drift is a test failure).  Same contract,
general over the record fields:

    {"classes": {"X": "Class X, ...", ...},          # optional: section titles, in order
     "columns": ["id", "statement", "sites", ...],    # optional: table columns
     "records": [{"id": "X1", "class": "X", "status": "OPEN", ...}, ...]}

Records are grouped by ``class`` (in the order of ``classes``, else first appearance),
each group gets a heading, a "k of n closed" line (status FIXED or BOUND counts as
closed) and one table row per record; list values are joined with "; " and cells are
escaped (pipes, newlines).

    python -m sigma0_b200.pipeline.register REGISTER.json DOC.md          # rewrite the section
    python -m sigma0_b200.pipeline.register REGISTER.json DOC.md --check  # exit 1 if stale
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import Dict, List

BEGIN = "<!-- REGISTER:BEGIN -->"
END = "<!-- REGISTER:END -->"
CLOSED = ("FIXED", "BOUND")


def _cell(v) -> str:
    if isinstance(v, bool):
        v = "**yes**" if v else "no"
    elif isinstance(v, (list, tuple)):
        v = "; ".join(f"`{x}`" for x in v)
    return str(v).replace("|", "\\|").replace("\n", " ").strip()


def render(reg: Dict) -> str:
    recs: List[Dict] = reg.get("records") or reg.get("defects") or []
    titles: Dict[str, str] = reg.get("classes", {})
    order = list(titles) + [c for c in dict.fromkeys(r["class"] for r in recs) if c not in titles]
    cols = reg.get("columns") or [k for k in recs[0] if k != "class"] if recs else []
    out: List[str] = []
    for cls in order:
        rows = [r for r in recs if r["class"] == cls]
        if not rows:
            continue
        closed = sum(r.get("status") in CLOSED for r in rows)
        out += [f"### {titles.get(cls, 'Class ' + cls)}", "", f"{closed} of {len(rows)} closed.", "",
                "| " + " | ".join(cols) + " |", "|" + "---|" * len(cols)]
        for r in rows:
            cells = []
            for c in cols:
                v = _cell(r.get(c, ""))
                cells.append(f"**{v}**" if c == "id" or (c == "status" and r.get(c) in CLOSED) else v)
            out.append("| " + " | ".join(cells) + " |")
        out.append("")
    return "\n".join(out)


def splice(text: str, body: str) -> str:
    i, j = text.index(BEGIN), text.index(END)
    if j < i:
        raise ValueError("the END marker precedes the BEGIN marker")
    return text[:i + len(BEGIN)] + "\n\n" + body + "\n" + text[j:]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("register")
    ap.add_argument("document")
    ap.add_argument("--check", action="store_true")
    a = ap.parse_args(argv)
    with open(a.register) as f:
        reg = json.load(f)
    with open(a.document) as f:
        cur = f.read()
    new = splice(cur, render(reg))
    if a.check:
        if new != cur:
            print(f"{a.document} is out of date with {a.register}", file=sys.stderr)
            return 1
        print("register section is up to date")
        return 0
    with open(a.document, "w") as f:
        f.write(new)
    print(f"rendered {len(reg.get('records') or reg.get('defects') or [])} records into {a.document}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
