"""Build recipe for the CPU oracle (test infrastructure).

Compiles oracle/nsrl_oracle.cpp into oracle/liboracle.so with g++.  Only the
tests, the smoke check and the CPU-baseline leg of bench.py load the result.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = [os.path.join(HERE, "nsrl_oracle.cpp")]
HDR = [os.path.join(HERE, "nsrl_oracle.hpp")]
OUT = os.path.join(HERE, "liboracle.so")


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(p) > t for p in SRC + HDR)


def build(force: bool = False) -> str:
    if force or needs_build():
        tmp = f"{OUT}.{os.getpid()}.tmp"  # one temporary per process: ranks may build at once
        cmd = ["g++", "-std=c++17", "-O3", "-fPIC", "-shared", "-pthread", "-Wall", "-o", tmp] + SRC
        subprocess.check_call(cmd)
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))


NATIVE_OUT = os.path.join(HERE, "liboracle_native.so")


def build_native() -> str:
    """Same sources with -march=native for timing the CPU baseline on the host it runs on."""
    if not os.path.exists(NATIVE_OUT) or os.path.getmtime(NATIVE_OUT) < max(os.path.getmtime(p) for p in SRC + HDR):
        tmp = f"{NATIVE_OUT}.{os.getpid()}.tmp"
        cmd = ["g++", "-std=c++17", "-O3", "-march=native", "-fPIC", "-shared", "-pthread", "-o", tmp] + SRC
        try:
            subprocess.check_call(cmd)
        except (subprocess.CalledProcessError, OSError):
            return build()
        os.replace(tmp, NATIVE_OUT)
    return NATIVE_OUT
