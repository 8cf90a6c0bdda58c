"""Build the reference's own Metal Adam kernel as a CPU checker library.

Reads ``src/mlx_extensions.cpp`` where it lies under the reference checkout,
extracts the MSL source string of ``fused_adam_step`` (src/mlx_extensions.cpp:98-153)
into ``oracle/_ref/ref_fused_adam_step.inc`` and compiles it, with
``oracle/msl_prelude.h`` force-included and ``oracle/ref_adam_driver.cpp`` as
the driver, into ``oracle/_ref/libref_adam.so``.  Nothing under ``oracle/_ref``
is committed.  TEST INFRASTRUCTURE ONLY.

Usage: ``python oracle/build_ref.py REFERENCE_ROOT``.
Returns quietly without building when the reference checkout is absent.
"""
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_root: str) -> bool:
    src = os.path.join(ref_root, "src", "mlx_extensions.cpp")
    if not os.path.exists(src):
        return False
    text = open(src).read()
    m = re.search(r'R"\((.*?)\)"', text, re.S)
    if m is None or "fused_adam_step" not in m.group(1):
        raise RuntimeError("could not find the MSL fused_adam_step source in " + src)
    body = m.group(1).replace("#include <metal_stdlib>", "")
    os.makedirs(OUT, exist_ok=True)
    with open(os.path.join(OUT, "ref_fused_adam_step.inc"), "w") as f:
        f.write(body)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-Wno-attributes",
           "-I", HERE, "-I", OUT, "-include", os.path.join(HERE, "msl_prelude.h"),
           os.path.join(HERE, "ref_adam_driver.cpp"), "-o", os.path.join(OUT, "libref_adam.so")]
    subprocess.check_call(cmd)
    return True


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/build_ref.py REFERENCE_ROOT")
    ok = build(sys.argv[1])
    print("built oracle/_ref/libref_adam.so" if ok else "reference checkout absent; nothing built")
