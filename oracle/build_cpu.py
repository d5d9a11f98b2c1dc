"""Build the CPU restatement ``oracle/_build/libswarp_cpu.so`` (gcc, OpenMP).

Test infrastructure / CPU baseline only. ``-ffp-contract=off`` keeps every multiply and
add rounded as written (no FMA contraction), as in the restated reference arithmetic.
"""

from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(OUT, "libswarp_cpu.so")
SRC = os.path.join(HERE, "cpu_port.c")
CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-std=c11"]


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cc = shutil.which("gcc") or "gcc"
    os.makedirs(OUT, exist_ok=True)
    objs = []
    for real, sfx in (("float", "f32"), ("double", "f64")):
        obj = os.path.join(OUT, f"cpu_port_{sfx}.o")
        subprocess.run([cc, *CFLAGS, f"-DREAL={real}", f"-DSFX(n)=n##_{sfx}", "-c", SRC, "-o", obj],
                       check=True)
        objs.append(obj)
    subprocess.run([cc, "-shared", "-fopenmp", "-o", LIB + ".tmp", *objs, "-lm"], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
