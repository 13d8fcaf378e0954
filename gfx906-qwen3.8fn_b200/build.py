"""Build libqwen_moe_b200.so in-tree with nvcc for sm_100a.

Usage: python gfx906-qwen3.8fn_b200/build.py [--verbose-ptxas]
The library is written next to this file; it is git-ignored but travels with
the repository snapshot to the GPU machines.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqwen_moe_b200.so")
SOURCES = ["moe_layer.cu", "route_groups.cpp"]
HEADERS = ["common.cuh", "expert_kernels.cuh", "route_kernels.cuh", "stream_kernels.cuh", "ptx.cuh", "tc_kernels.cuh",
           "tcr_kernels.cuh",
           "ep_kernels.cuh", "ep_common.cuh", "router_kernels.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-DQMOE_BUILD"]


def _inputs():
    paths = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    paths.append(os.path.join(HERE, "..", "include", "qwen_moe_b200.h"))
    paths.append(os.path.join(HERE, "..", "include", "qmoe", "routes.hpp"))
    paths.append(os.path.join(CSRC, "expf_table.c"))
    paths.append(os.path.abspath(__file__))
    return paths


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _inputs() if os.path.exists(p))


def expf_table_object(build_dir):
    """Object file holding the C library's expf corrections (csrc/expf_table.c):
    generated once by running that program, embedded with .incbin."""
    table = os.path.join(build_dir, "expf_table.bin")
    gen = os.path.join(build_dir, "expf_table")
    src = os.path.join(CSRC, "expf_table.c")
    if not os.path.exists(table) or os.path.getmtime(table) < os.path.getmtime(src):
        subprocess.run(["gcc", "-O2", src, "-o", gen, "-lm"], check=True)
        subprocess.run([gen, table + ".tmp"], check=True, stdout=subprocess.DEVNULL)
        os.replace(table + ".tmp", table)
    asm = os.path.join(build_dir, "expf_table.S")
    with open(asm, "w") as f:
        f.write('\t.section .rodata\n\t.balign 16\n'
                '\t.globl qmoe_expf_table_begin\n\t.hidden qmoe_expf_table_begin\nqmoe_expf_table_begin:\n'
                f'\t.incbin "{table}"\n'
                '\t.globl qmoe_expf_table_end\n\t.hidden qmoe_expf_table_end\nqmoe_expf_table_end:\n'
                '\t.section .note.GNU-stack,"",@progbits\n')
    obj = os.path.join(build_dir, "expf_table.o")
    subprocess.run(["gcc", "-c", asm, "-o", obj], check=True)
    return obj


def build(force=False, ptxas_verbose=False):
    if not force and not stale():
        return LIB
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(build_dir, os.path.splitext(src)[0] + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        subprocess.run(cmd, check=True)
        objs.append(obj)
    objs.append(expf_table_object(build_dir))
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"],
                   check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, ptxas_verbose="--verbose-ptxas" in sys.argv)
    print(LIB)
