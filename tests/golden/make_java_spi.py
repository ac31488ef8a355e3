"""Writes tests/golden/java_spi.json: the signatures of the reference's engine
SPI that the Java drop-in (java/nablatensor-engine-b200) compiles against.

Run from the repository root where the reference sources are present:

    python tests/golden/make_java_spi.py /path/to/nablatensor

For each class it records the methods (name, parameter types, return type,
modifiers) and public fields declared at class level, and the AadOpEnum
constants in ordinal order.  tests/test_java_dropin.py checks the drop-in's
overrides, calls and op-code mapping against this file, so the test needs
no reference checkout.
"""
import json
import os
import re
import sys

CLASSES = {
    "AadEngine": "nablatensor-core/src/main/java/com/nablatensor/engine/AadEngine.java",
    "AadExecutable": "nablatensor-core/src/main/java/com/nablatensor/engine/AadExecutable.java",
    "AbstractAadExecutable": "nablatensor-core/src/main/java/com/nablatensor/engine/AbstractAadExecutable.java",
    "GpuAadExecutable": "nablatensor-core/src/main/java/com/nablatensor/engine/GpuAadExecutable.java",
    "AadTape": "nablatensor-core/src/main/java/com/nablatensor/engine/AadTape.java",
    "FlatTape": "nablatensor-core/src/main/java/com/nablatensor/engine/FlatTape.java",
    "AadOptions": "nablatensor-core/src/main/java/com/nablatensor/engine/AadOptions.java",
    "AadTotals": "nablatensor-core/src/main/java/com/nablatensor/engine/AadTotals.java",
    "AadResult": "nablatensor-core/src/main/java/com/nablatensor/engine/AadResult.java",
}
ENUM = "nablatensor-core/src/main/java/com/nablatensor/engine/AadOpEnum.java"

MODS = {"public", "protected", "private", "static", "final", "default", "abstract", "synchronized"}
METHOD = re.compile(r"^  (?=\S)((?:(?:public|protected|private|static|final|default|abstract|synchronized)\s+)*)"
                    r"([\w<>\[\], ?.]+?)\s+(\w+)\s*\(([^)]*)\)")
FIELD = re.compile(r"^  (?=\S)((?:(?:public|protected|private|static|final)\s+)+)([\w<>\[\], ?.]+?)\s+(\w+)\s*[;=]")


def _strip(text):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _params(p):
    """Parameter types of a declaration, split at top-level commas (generic
    arguments may hold commas of their own)."""
    parts, depth, cur = [], 0, ""
    for ch in p:
        depth += ch == "<"
        depth -= ch == ">"
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    parts.append(cur)
    out = []
    for part in [x.strip() for x in parts if x.strip()]:
        part = re.sub(r"^final\s+", "", part)
        out.append(re.sub(r"\s+\w+$", "", part).replace(" ", ""))
    return out


def parse(path):
    methods, fields = [], []
    for line in _strip(open(path).read()).splitlines():
        m = METHOD.match(line)
        if m and m.group(3) not in ("if", "for", "while", "switch", "return", "new"):
            mods = m.group(1).split()
            methods.append({"name": m.group(3), "params": _params(m.group(4)), "returns": m.group(2).strip(),
                            "modifiers": sorted(mods)})
            continue
        f = FIELD.match(line)
        if f:
            fields.append({"name": f.group(3), "type": f.group(2).strip(), "modifiers": sorted(f.group(1).split())})
    return methods, fields


def main(root):
    out = {"classes": {}}
    for name, rel in CLASSES.items():
        methods, fields = parse(os.path.join(root, rel))
        out["classes"][name] = {"source": rel, "methods": methods, "fields": fields}
    text = _strip(open(os.path.join(root, ENUM)).read())
    body = text[text.index("{") + 1:]
    body = body[:body.index(";")] if ";" in body else body[:body.index("}")]
    out["AadOpEnum"] = [c.strip().split("(")[0] for c in body.split(",") if c.strip()]
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "java_spi.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print(dst)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else ".")
