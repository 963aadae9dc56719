"""Build libfkv.so (sm_100a) in-tree: ``python -m foveated_kv_b200.build``."""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose: bool = False, jobs: int = 8) -> str:
    csrc = os.path.join(HERE, "csrc")
    cmd = ["make", "-C", csrc, f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"libfkv build failed:\n{res.stdout}\n{res.stderr}")
    return os.path.join(HERE, "_lib", "libfkv.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
