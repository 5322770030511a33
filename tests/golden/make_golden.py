"""Extracts the known-answer vectors of the reference's own unit tests into
reference_kats.json. Run it where a rustyneedle checkout is at hand, giving the
checkout's root as the first argument or in $RUSTYNEEDLE_REFERENCE; the JSON is
committed so the tests never read the reference at run time.

    python tests/golden/make_golden.py <rustyneedle checkout>

Sources (paths inside the rustyneedle workspace):
  crates/model/tests/ladder.rs      bisection order and depth selections
  crates/model/tests/depth.rs       the depth-8 layer set
  crates/kernels/tests/walsh.rs     transform sizes, input formula, tolerance
  crates/kernels/tests/kronecker.rs 32x32 input formula and tolerance
  crates/kernels/tests/softmax.rs   fast_exp range/tolerance and softmax logits
  crates/model/tests/prefill.rs     batched-vs-stepped cosine threshold
"""

from __future__ import annotations

import json
import os
import re
import sys

ROOT = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RUSTYNEEDLE_REFERENCE")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")


def read(path: str) -> str:
    with open(os.path.join(ROOT, path)) as f:
        return f.read()


def ints(text: str) -> list[int]:
    return [int(x) for x in re.findall(r"-?\d+", text)]


def main() -> None:
    if not ROOT:
        sys.exit("usage: make_golden.py <rustyneedle checkout> (or set RUSTYNEEDLE_REFERENCE)")
    ladder = read("crates/model/tests/ladder.rs")
    order = ints(re.search(r"ladder::order\(20\),\s*vec!\[([^\]]*)\]", ladder).group(1))
    selects = {}
    for depth, body in re.findall(r"ladder::select\(20,\s*(\d+)\)\.unwrap\(\),\s*vec!\[([^\]]*)\]", ladder):
        selects[depth] = ints(body)
    if re.search(r"ladder::select\(20,\s*20\)\.unwrap\(\),\s*\(0\.\.20\)", ladder):
        selects["20"] = list(range(20))
    small = re.search(r"ladder::select\(8,\s*2\)\.unwrap\(\),\s*vec!\[([^\]]*)\]", ladder)
    rejects = [[int(a), int(b)] for a, b in re.findall(r"ladder::select\((\d+),\s*(\d+)\)\.is_none\(\)", ladder)]

    depth = read("crates/model/tests/depth.rs")
    depth8 = ints(re.search(r"active_layers\(\),\s*&\[([^\]]*)\]", depth).group(1))

    walsh = read("crates/kernels/tests/walsh.rs")
    sizes = ints(re.search(r"for size in \[([^\]]*)\]", walsh).group(1))
    wf = re.search(r"\(\(\(i \* (\d+) \+ size\) % (\d+)\) as f32 - ([\d.]+)\) / ([\d.]+)", walsh)
    wtol = float(re.search(r"worst < ([\d.e-]+)", walsh).group(1))

    kron = read("crates/kernels/tests/kronecker.rs")
    kf = re.search(r"\(\(\(i \* (\d+) \+ seed \* (\d+)\) % (\d+)\) as f32 - ([\d.]+)\) / ([\d.]+)", kron)
    kseeds = ints(re.search(r"\(make\((\d+)\),\s*make\((\d+)\),\s*make\((\d+)\)\)", kron).group(0))
    ktol = float(re.search(r"worst < ([\d.e-]+)", kron).group(1))

    soft = read("crates/kernels/tests/softmax.rs")
    frange = re.search(r"let mut x = (-?[\d.]+)f32;\s*while x <= ([\d.]+) \{", soft)
    fstep = float(re.search(r"x \+= ([\d.]+);", soft).group(1))
    ftol = float(re.search(r"worst < ([\d.e-]+)", soft).group(1))
    logits = [float(x) for x in re.search(r"let logits = \[([^\]]*)\];", soft).group(1).replace("f32", "").split(",")]
    stol = float(re.search(r"exact\)\.abs\(\) < ([\d.e-]+)", soft).group(1))

    prefill = read("crates/model/tests/prefill.rs")
    pcos = float(re.search(r"cosine\(&a, &b\) > ([\d.]+)", prefill).group(1))
    htol = float(re.search(r"\(ha - hb\)\.abs\(\) < ([\d.]+)", prefill).group(1))
    dcos = float(re.search(r"cosine\(&a\.logits\(\), &b\.logits\(\)\) > ([\d.]+)", depth).group(1))

    kats = {
        "source": "rustyneedle crates/{model,kernels}/tests (see make_golden.py)",
        "ladder_order_20": order,
        "ladder_select_20": selects,
        "ladder_select_8_2": ints(small.group(1)),
        "ladder_rejects": rejects,
        "depth8_layers": depth8,
        "walsh": {"sizes": sizes, "mul": int(wf.group(1)), "mod": int(wf.group(2)), "offset": float(wf.group(3)),
                  "div": float(wf.group(4)), "tolerance": wtol},
        "kronecker": {"mul": int(kf.group(1)), "seed_mul": int(kf.group(2)), "mod": int(kf.group(3)),
                      "offset": float(kf.group(4)), "div": float(kf.group(5)), "seeds": kseeds, "size": 32,
                      "tolerance": ktol},
        "fast_exp": {"start": float(frange.group(1)), "stop": float(frange.group(2)), "step": fstep,
                     "tolerance": ftol},
        "softmax": {"logits": logits, "tolerance": stol},
        "prefill_cosine": pcos,
        "prefill_head_tolerance": htol,
        "full_depth_cosine": dcos,
    }
    with open(OUT, "w") as f:
        json.dump(kats, f, indent=1)
    print(OUT)


if __name__ == "__main__":
    main()
