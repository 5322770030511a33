"""Extracts the tool schemas of the reference's example tool files
(examples/tools/*.json in a rustyneedle checkout) into tool_schemas.json: per
file, each tool's name and parameters (descriptions dropped), the input
CallGrammar::from_tools_json reads. Run it where a checkout is at hand, giving
its root as the first argument or in $RUSTYNEEDLE_REFERENCE; the JSON is
committed so the tests never read the reference at run time.

    python tests/golden/make_tool_schemas.py <rustyneedle checkout>
"""

from __future__ import annotations

import glob
import json
import os
import sys

ROOT = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RUSTYNEEDLE_REFERENCE")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tool_schemas.json")


def strip(schema):
    """The schema without its human-readable descriptions; the keys of a
    "properties" map are property names and stay."""
    if isinstance(schema, dict):
        out = {}
        for k, v in schema.items():
            if k == "description" and isinstance(v, str):
                continue
            if k in ("properties", "$defs", "definitions") and isinstance(v, dict):
                out[k] = {name: strip(child) for name, child in v.items()}
            else:
                out[k] = strip(v)
        return out
    if isinstance(schema, list):
        return [strip(v) for v in schema]
    return schema


def main() -> None:
    if not ROOT:
        sys.exit("usage: make_tool_schemas.py <rustyneedle checkout> (or set RUSTYNEEDLE_REFERENCE)")
    out = {}
    for path in sorted(glob.glob(os.path.join(ROOT, "examples", "tools", "*.json"))):
        with open(path) as f:
            tools = json.load(f)
        kept = []
        for tool in tools:
            fn = tool.get("function", tool)
            entry = {"name": fn["name"]}
            if "parameters" in fn:
                entry["parameters"] = strip(fn["parameters"])
            kept.append(entry)
        out[os.path.basename(path)] = kept
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
    print(OUT)


if __name__ == "__main__":
    main()
