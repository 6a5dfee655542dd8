"""Builds libbloom_ffi.so (the C ABI of csrc/ffi/bloom.h) in-tree.

    python csrc/ffi/build.py            # -> bloom_b200/ffi/libbloom_ffi.so

The library embeds the Python interpreter it was built against (libpython
from sysconfig) and imports bloom_b200 from the repository root, which it
adds to sys.path through PYTHONPATH or the host's own path.
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(ROOT, "bloom_b200", "ffi", "libbloom_ffi.so")


def build(out: str = OUT) -> str:
    inc = sysconfig.get_config_var("INCLUDEPY")
    libdir = sysconfig.get_config_var("LIBDIR")
    ver = sysconfig.get_config_var("LDVERSION") or sysconfig.get_config_var("VERSION")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
           f"-I{inc}", f"-I{HERE}", os.path.join(HERE, "bloom_ffi.cpp"), "-o", out,
           f"-L{libdir}", f"-lpython{ver}", f"-Wl,-rpath,{libdir}"]
    subprocess.check_call(cmd)
    return out


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else OUT))
