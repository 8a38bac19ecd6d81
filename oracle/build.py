"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``dz_oracle.cpp`` into ``oracle/libdzoracle.so`` with the flags that
make it follow the Rust reference bit for bit on the same CPU:
``-mavx2 -mfma -mf16c`` (same intrinsics) and ``-ffp-contract=off`` (rustc never fuses
a separate multiply and add).

The reference itself (Rust, Cargo workspace) cannot be compiled here: there is
no cargo/rustc in the image, so there is no ``oracle/_ref`` build.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "dz_oracle.cpp")
OUT = os.path.join(HERE, "libdzoracle.so")


def build(force: bool = False) -> str:
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= os.path.getmtime(SRC)):
        return OUT
    cmd = ["g++", "-O2", "-std=c++17", "-mavx2", "-mfma", "-mf16c", "-ffp-contract=off",
           "-fno-fast-math", "-fPIC", "-shared", "-pthread", SRC, "-o", OUT + ".tmp"]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
