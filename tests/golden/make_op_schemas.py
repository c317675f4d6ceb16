"""Extract the reference's torch op schemas into tests/golden/op_schemas.json.

Reads the TORCH_LIBRARY(dbs, ...) block of the reference's
python/torch_extension.cpp (the m.def strings of final_scores_forward and
final_scores_backward) from the reference source tree: the directory given
as the first argument, else DBS_REFERENCE_DIR, else the tree beside this
checkout (../reference from the repository root, as oracle/Makefile uses).

    python tests/golden/make_op_schemas.py [REFERENCE_DIR]
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main(argv):
    ref = argv[1] if len(argv) > 1 else os.environ.get("DBS_REFERENCE_DIR",
                                                       os.path.join(os.path.dirname(ROOT), "reference"))
    src = open(os.path.join(ref, "python", "torch_extension.cpp")).read()
    block = re.search(r"TORCH_LIBRARY\(dbs,\s*m\)\s*\{(.*?)\n\}", src, flags=re.S)
    if block is None:
        raise SystemExit("TORCH_LIBRARY(dbs, m) block not found")
    schemas = re.findall(r'm\.def\("([^"]+)"\)', block.group(1))
    out = {"source": "python/torch_extension.cpp, TORCH_LIBRARY(dbs, m)", "schemas": schemas}
    with open(os.path.join(HERE, "op_schemas.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(f"{len(schemas)} schemas")


if __name__ == "__main__":
    main(sys.argv)
