"""Build libbeacon_cuda.so (and nothing else) with the package Makefile."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", "-C", HERE, f"-j{jobs}"], check=True)
    return os.path.join(HERE, "lib", "libbeacon_cuda.so")


if __name__ == "__main__":
    print(build(int(sys.argv[1]) if len(sys.argv) > 1 else 8))
