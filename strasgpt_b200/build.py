"""Build the in-tree libraries (nvcc cross-compiles sm_100a without a GPU)."""
import os
import subprocess

from . import _paths


def build(jobs: int = 8, verbose: bool = False) -> None:
    """make -C strasgpt_b200/csrc: libstrasgpt.so and libstrasgpt_synth.so."""
    cmd = ["make", "-C", _paths.CSRC, f"-j{jobs}"]
    out = subprocess.run(cmd, capture_output=not verbose, text=True)
    if out.returncode != 0:
        raise RuntimeError("build failed:\n" + (out.stdout or "") + (out.stderr or ""))
    for p in (_paths.main_lib(), _paths.synth_lib()):
        if not os.path.exists(p):
            raise RuntimeError(f"build did not produce {p}")


if __name__ == "__main__":
    build(verbose=True)
