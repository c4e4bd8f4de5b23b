"""Regenerates tests/golden/merge.json from the REFERENCE's own merge script.

    python tests/golden/make_merge_golden.py [REFERENCE_ROOT]   (or TB_REFERENCE_DIR=...)

Builds the shard directories of tests/inputs.merge_tree() in a fresh temporary
tree for each run of tests/inputs.MERGE_RUNS, runs the reference's
scripts/merge_tbm.py there, and records its exit code, its stdout and the
sha256 and size of the container it wrote.  The reference tree is needed only
to run this script; tests/test_merge.py checks the native tb-merge against the
committed fixture on any machine.
"""
import hashlib
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import inputs  # noqa: E402

# The reference checkout: TB_REFERENCE_DIR, else the first argument, else the
# default mount point of this build's container.
REF_ROOT = os.environ.get("TB_REFERENCE_DIR") or (sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
SCRIPT = os.path.join(REF_ROOT, "scripts", "merge_tbm.py")


def output_arg(args):
    return args[args.index("--output") + 1]


def main():
    out = {"generator": "tests/golden/make_merge_golden.py (the reference's scripts/merge_tbm.py)"}
    for key, (args, cwd) in inputs.MERGE_RUNS.items():
        with tempfile.TemporaryDirectory() as d:
            inputs.merge_tree(d)
            run_dir = os.path.join(d, cwd)
            r = subprocess.run([sys.executable, SCRIPT, *args], cwd=run_dir, capture_output=True, text=True)
            path = os.path.join(run_dir, output_arg(args))
            rec = {"returncode": r.returncode, "stdout": r.stdout}
            if os.path.exists(path):
                data = open(path, "rb").read()
                rec["sha256"] = hashlib.sha256(data).hexdigest()
                rec["size"] = len(data)
                n = int.from_bytes(data[-4:], "little")
                rec["index"] = json.loads(data[-4 - n:-4].decode("utf-8"))
            out[key] = rec
    with open(os.path.join(HERE, "merge.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True, ensure_ascii=True)
    print("wrote merge.json")


if __name__ == "__main__":
    main()
