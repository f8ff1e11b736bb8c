"""Build recipe for the CPU oracle (test infrastructure, see h3_oracle.c).

Compiles oracle/h3_oracle.c into oracle/liboracle.so with gcc.  The flags keep
every binary32 operation separate (-ffp-contract=off) and avoid -ffast-math so
that the restatement follows IEEE rounding exactly; the code is baseline
x86-64 (no -march) so the library runs on any host it is copied to.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "h3_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")


def build_oracle(force=False):
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
           "-Wall", "-Wextra", "-o", LIB + ".tmp", SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build_oracle(force=True))
