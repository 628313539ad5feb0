"""Build recipe for the CPU oracle (test infrastructure, not the product).

Compiles ``popcorn_oracle.cpp`` into ``oracle/_build/libpopcorn_oracle.so``
with g++ and OpenMP. The reference itself (Swift + Metal) cannot be built on
Linux, so there is no ``oracle/_ref`` library; the restatement in
``popcorn_oracle.cpp`` is the oracle.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "popcorn_oracle.cpp")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libpopcorn_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["g++", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-std=c++17",
           "-o", LIB, SRC]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
