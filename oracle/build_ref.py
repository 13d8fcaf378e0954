#!/usr/bin/env python3
"""Build the reference's own CPU path into oracle/_ref/ (test infrastructure).

Compiles, directly from the reference sources where they lie (--ref DIR, else
$QWEN_REF_DIR, else a checkout named "reference" beside this repository), with
g++ and no build system:

* oracle/_ref/bin/{routes,quant,cpu_expert}_test -- the reference's own CPU tests,
  run by --run-tests as the pin of the reference build itself;
* oracle/_ref/libqwen_ref_native.so -- oracle/ref_shim.cpp + src/routes.cpp,
  src/quant.cpp, src/model.cpp, src/cpu_expert.cpp at the reference's own
  expert shape (hidden 2560, intermediate 640);
* oracle/_ref/libqwen_ref.so -- the same, with CpuExpert shape-patched to
  hidden 2048 / intermediate 512 (the shapes this repository benchmarks).

The shape patch is applied to a copy of src/cpu_expert.{hpp,cpp} in a temporary
directory (never written into the repository); every replacement is an exact
string match that must occur exactly once, so a changed reference fails loudly.
Outputs go only into oracle/_ref/, which is git-ignored.
"""
import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
FLAGS = ["-std=c++20", "-O2", "-ffp-contract=off", "-pthread", "-fPIC"]

# (file, old, new): src/cpu_expert.cpp:66-80,91-92,224-245 and src/cpu_expert.hpp:62-67
# hard-wire hidden 2560 / intermediate 640; these replacements retarget 2048 / 512.
PATCHES = [
    ("cpu_expert.cpp", "m.input != (down ? 640 : 2560) || m.output != (down ? 2560 : 640)",
     "m.input != (down ? 512 : 2048) || m.output != (down ? 2048 : 512)"),
    ("cpu_expert.cpp", "constexpr std::size_t blocks = 51200;", "constexpr std::size_t blocks = 32768;"),
    ("cpu_expert.cpp", "job.stage == CpuExpertStage::gate_up ? 1280 : 2560;",
     "job.stage == CpuExpertStage::gate_up ? 1024 : 2048;"),
    ("cpu_expert.cpp", "job.stage == CpuExpertStage::down ? 20 : 80;",
     "job.stage == CpuExpertStage::down ? 16 : 64;"),
    ("cpu_expert.cpp",
     "scratch.middle_q8.data() + std::size_t(c) * 20, job.input[std::size_t(c)].data(), 20 * sizeof(Q8_1)",
     "scratch.middle_q8.data() + std::size_t(c) * 16, job.input[std::size_t(c)].data(), 16 * sizeof(Q8_1)"),
    ("cpu_expert.cpp",
     "scratch.gathered_x.data() + std::size_t(c) * 80, job.input[std::size_t(c)].data(), 80 * sizeof(Q8_1)",
     "scratch.gathered_x.data() + std::size_t(c) * 64, job.input[std::size_t(c)].data(), 64 * sizeof(Q8_1)"),
    ("cpu_expert.cpp", "const auto middle_size = std::size_t(job.columns) * 640;",
     "const auto middle_size = std::size_t(job.columns) * 512;"),
    ("cpu_expert.cpp",
     "std::memcpy(job.output.data() + std::size_t(c) * 1280, scratch.gate.data() + std::size_t(c) * 640, 640 * sizeof(float));",
     "std::memcpy(job.output.data() + std::size_t(c) * 1024, scratch.gate.data() + std::size_t(c) * 512, 512 * sizeof(float));"),
    ("cpu_expert.cpp",
     "std::memcpy(job.output.data() + std::size_t(c) * 1280 + 640, scratch.up.data() + std::size_t(c) * 640, 640 * sizeof(float));",
     "std::memcpy(job.output.data() + std::size_t(c) * 1024 + 512, scratch.up.data() + std::size_t(c) * 512, 512 * sizeof(float));"),
    ("cpu_expert.hpp", "std::array<Q8_1, 240> gathered_x;", "std::array<Q8_1, 192> gathered_x;"),
    ("cpu_expert.hpp", "std::array<Q8_1, 60> middle_q8;", "std::array<Q8_1, 48> middle_q8;"),
    ("cpu_expert.hpp", "std::array<float, 1920> gate, up, middle;", "std::array<float, 1536> gate, up, middle;"),
    ("cpu_expert.hpp", "std::array<float, 7680> down;", "std::array<float, 6144> down;"),
]


def run(cmd, **kw):
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, **kw)


def patched_tree(ref_src, tmp):
    for name in ("cpu_expert.cpp", "cpu_expert.hpp"):
        shutil.copy(os.path.join(ref_src, name), os.path.join(tmp, name))
    for name, old, new in PATCHES:
        path = os.path.join(tmp, name)
        text = open(path).read()
        count = text.count(old)
        if count != 1:
            raise SystemExit(f"shape patch: expected exactly one match in {name} for {old!r}, found {count}")
        open(path, "w").write(text.replace(old, new))
    return tmp


def build(ref, run_tests):
    src = os.path.join(ref, "src")
    if not os.path.isfile(os.path.join(src, "cpu_expert.cpp")):
        raise SystemExit(f"reference sources not found under {ref}")
    os.makedirs(os.path.join(OUT, "bin"), exist_ok=True)
    common = [os.path.join(src, f) for f in ("routes.cpp", "quant.cpp", "model.cpp")]
    shim = os.path.join(HERE, "ref_shim.cpp")
    cxx = os.environ.get("CXX", "g++")
    # native-shape shim
    run([cxx, *FLAGS, "-shared", "-I", src, shim, *common, os.path.join(src, "cpu_expert.cpp"),
         "-o", os.path.join(OUT, "libqwen_ref_native.so")])
    # shape-patched shim: the patched header/source come first on the include path
    with tempfile.TemporaryDirectory() as tmp:
        patched_tree(src, tmp)
        run([cxx, *FLAGS, "-shared", "-I", tmp, "-I", src, shim, *common,
             os.path.join(tmp, "cpu_expert.cpp"), "-o", os.path.join(OUT, "libqwen_ref.so")])
    if run_tests:
        tests = os.path.join(ref, "tests")
        for name, extra in (("routes", []), ("quant", []), ("cpu_expert", ["cpu_expert.cpp"])):
            exe = os.path.join(OUT, "bin", f"{name}_test")
            srcs = [os.path.join(tests, f"{name}_test.cpp"), *common] + [os.path.join(src, e) for e in extra]
            if name == "cpu_expert":
                srcs = [os.path.join(tests, "cpu_expert_test.cpp"), *common, os.path.join(src, "cpu_expert.cpp")]
            run([cxx, *[f for f in FLAGS if f != "-fPIC"], "-I", src, *srcs, "-o", exe])
            out = subprocess.run([exe], capture_output=True, text=True)
            tail = (out.stdout + out.stderr).strip().splitlines()[-1:]
            print(f"{name}_test exit={out.returncode}: {tail}")
            if out.returncode != 0:
                raise SystemExit(f"reference {name}_test failed")


def default_ref_tree():
    """$QWEN_REF_DIR, else the reference checkout beside this repository."""
    env = os.environ.get("QWEN_REF_DIR")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=default_ref_tree())
    ap.add_argument("--run-tests", action="store_true", help="also build and run the reference's CPU tests")
    args = ap.parse_args()
    if not os.path.isdir(args.ref):
        print(f"reference tree {args.ref} absent; keeping prebuilt oracle/_ref", file=sys.stderr)
        return 0
    build(args.ref, args.run_tests)
    return 0


if __name__ == "__main__":
    sys.exit(main())
