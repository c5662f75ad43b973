"""Extract the reference's known-answer vectors into tests/golden/vag_goldens.json
and tests/golden/optim_goldens.json.

Reads the reference's own test files as text (they are YAML / Markdown, no
reference code is executed):
  sheaf/tests/vag_tests.yaml:5-169         finite-difference value-and-grad goldens
  sheaf/tests/interpreter_tests.yaml:753-762  MLP value-and-grad loss with splitmix inputs
  README.md:33-43                          mse-loss value-and-grad example
  sheaf/tests/interpreter_tests.yaml:623-628  adamw-step with and without decay

Run from the repo root:  python tests/golden/make_goldens.py <reference_root>
(the directory holding the reference's sheaf/ and README.md).
"""
import json
import os
import re
import sys

if len(sys.argv) != 2:
    raise SystemExit("usage: python tests/golden/make_goldens.py <reference_root>")
REF = sys.argv[1]
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "vag_goldens.json")
OUT_OPTIM = os.path.join(os.path.dirname(os.path.abspath(__file__)), "optim_goldens.json")

NUM = r"[-+]?(?:\d+\.?\d*|\.\d+)(?:[eE][-+]?\d+)?"


def parse_value(s):
    """Parse Sheaf's printed value ("[33.0, [1. 1.]]") into nested lists."""
    toks = re.findall(NUM + r"|\[|\]", s)
    pos = 0

    def rd():
        nonlocal pos
        t = toks[pos]
        pos += 1
        if t == "[":
            out = []
            while toks[pos] != "]":
                out.append(rd())
            pos += 1
            return out
        return float(t)
    return rd()


def yaml_cases(path):
    """Minimal reader for the reference's flat YAML list of {name, test, expected}."""
    cases, cur, key = [], None, None
    for line in open(path):
        m = re.match(r"^- name: (.*)$", line)
        if m:
            cur = {"name": m.group(1).strip()}
            cases.append(cur)
            key = None
            continue
        m = re.match(r"^  (test|expected): ?(.*)$", line)
        if m and cur is not None:
            key = m.group(1)
            cur[key] = m.group(2).strip()
            continue
        if key == "test" and line.startswith("    "):
            cur["test"] = (cur["test"] + " " + line.strip()).strip(" >")
    return cases


def main():
    out = {"source": {}, "cases": {}}
    vag = os.path.join(REF, "sheaf/tests/vag_tests.yaml")
    for c in yaml_cases(vag):
        exp = c.get("expected", "").strip('"')
        if exp.startswith("ERROR"):
            out["cases"][c["name"]] = {"test": c.get("test", ""), "error": exp}
            continue
        v = parse_value(exp)
        if isinstance(v, list) and len(v) == 2 and not isinstance(v[0], list):
            out["cases"][c["name"]] = {"test": c.get("test", ""), "loss": v[0], "grad": v[1]}
    out["source"]["vag"] = "sheaf/tests/vag_tests.yaml"
    it = os.path.join(REF, "sheaf/tests/interpreter_tests.yaml")
    for c in yaml_cases(it):
        if c["name"] == "vag-mlp-loss":
            out["cases"]["vag-mlp-loss"] = {"test": c["test"], "loss": float(c["expected"].strip('"'))}
    out["source"]["mlp"] = "sheaf/tests/interpreter_tests.yaml"
    readme = open(os.path.join(REF, "README.md")).read()
    m = re.search(r"=> (\[0\.5 \[\[.*?\]\]\])", readme, re.S)
    v = parse_value(m.group(1))
    out["cases"]["readme-mse"] = {"test": "((value-and-grad (fn [W] (mse-loss (@ x W) y))) W)",
                                  "loss": v[0], "grad": v[1]}
    out["source"]["readme"] = "README.md"
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print(f"wrote {len(out['cases'])} cases to {OUT}")
    # (adamw-step p g m v t lr b1 b2 eps wd) on one-leaf trees {:w x}
    optim = {"source": "sheaf/tests/interpreter_tests.yaml", "cases": {}}
    for c in yaml_cases(it):
        if not c["name"].startswith("adamw-step"):
            continue
        leaves = [float(x) for x in re.findall(r"\{:w (" + NUM + r")\}", c["test"])]
        m = re.search(r"\(adamw-step p g m v ((?:" + NUM + r"\s*)+)\)", c["test"])
        args = [float(x) for x in m.group(1).split()]
        optim["cases"][c["name"]] = {"test": c["test"], "p": leaves[0], "g": leaves[1], "m": leaves[2],
                                     "v": leaves[3], "t": int(args[0]), "lr": args[1], "b1": args[2], "b2": args[3],
                                     "eps": args[4], "wd": args[5], "expected_p": float(c["expected"].strip('"'))}
    with open(OUT_OPTIM, "w") as f:
        json.dump(optim, f, indent=1, sort_keys=True)
    print(f"wrote {len(optim['cases'])} cases to {OUT_OPTIM}")


if __name__ == "__main__":
    main()
