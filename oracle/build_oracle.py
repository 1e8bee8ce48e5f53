"""Build recipe for the oracle's C library and, where the reference tree exists,
the reference-compiled checkers under oracle/_ref/.

TEST INFRASTRUCTURE ONLY (see oracle/hyp_oracle.c).

  * oracle/liboracle.so      <- oracle/hyp_oracle.c (gcc -O3 -fopenmp)
  * oracle/liboracle_rng.so  <- oracle/std_rng.cc (the standard library's mt19937_64 draw)
  * oracle/_ref/libref_index.so <- the reference's MLX-free sources
        native/hyperion_mlx/src/{kv.cc,geometry.cc,dispatch.cc}
    compiled where they lie, plus oracle/ref_shim.cc (a C wrapper of ours), so
    the tests can pin the ring/global index arithmetic and geometry validation
    against the reference's own code.
  * oracle/_ref/abi_contract_test <- the reference's
        native/hyperion_mlx/tests/abi_contract_test.cc
    compiled unchanged against this repository's include/hyperion_mlx.h and
    linked with hyperion_b200/libhyperion_mlx.so: the drop-in conformance test.
Outputs go only to oracle/ and oracle/_ref/ (both git-ignored build products).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
# The reference checkout: $HYPERION_REFERENCE_ROOT, else a directory named `reference`
# beside this repository's checkout. Without either, only the oracle's own libraries build.
REF = os.environ.get("HYPERION_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")
REF_SRC = os.path.join(REF, "native", "hyperion_mlx", "src")
REF_TESTS = os.path.join(REF, "native", "hyperion_mlx", "tests")
REF_INC = os.path.join(REF, "native", "hyperion_mlx", "include")


def _run(cmd):
    subprocess.run(cmd, check=True)


def build() -> str:
    out = os.path.join(HERE, "liboracle.so")
    src = os.path.join(HERE, "hyp_oracle.c")
    if not os.path.exists(out) or os.path.getmtime(out) < os.path.getmtime(src):
        _run(["gcc", "-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=c11",
              src, "-o", out + ".tmp", "-lm"])
        os.replace(out + ".tmp", out)
    rng_out = os.path.join(HERE, "liboracle_rng.so")
    rng_src = os.path.join(HERE, "std_rng.cc")
    if not os.path.exists(rng_out) or os.path.getmtime(rng_out) < os.path.getmtime(rng_src):
        _run(["g++", "-O2", "-fPIC", "-shared", "-std=c++17", rng_src, "-o", rng_out + ".tmp"])
        os.replace(rng_out + ".tmp", rng_out)
    return out


def reference_present() -> bool:
    return os.path.isfile(os.path.join(REF_SRC, "kv.cc"))


def build_ref(lib_path: str | None = None) -> dict:
    """Compile the reference's MLX-free sources and ABI contract test (needs the tree)."""
    built = {}
    if not reference_present():
        return built
    ref_dir = os.path.join(HERE, "_ref")
    os.makedirs(ref_dir, exist_ok=True)
    so = os.path.join(ref_dir, "libref_index.so")
    _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared",
          "-I", REF_SRC, "-I", REF_INC,
          os.path.join(REF_SRC, "kv.cc"), os.path.join(REF_SRC, "geometry.cc"),
          os.path.join(REF_SRC, "dispatch.cc"), os.path.join(HERE, "ref_shim.cc"),
          "-o", so])
    built["index"] = so
    lib_path = lib_path or os.path.join(REPO, "hyperion_b200", "libhyperion_mlx.so")
    if os.path.exists(lib_path):
        exe = os.path.join(ref_dir, "abi_contract_test")
        _run(["g++", "-std=c++17", "-O2", "-I", os.path.join(REPO, "include"),
              os.path.join(REF_TESTS, "abi_contract_test.cc"), "-o", exe,
              "-L", os.path.dirname(lib_path), "-lhyperion_mlx",
              "-Wl,-rpath," + os.path.dirname(lib_path)])
        built["abi_contract_test"] = exe
    return built


if __name__ == "__main__":
    print(build())
    print(build_ref(sys.argv[1] if len(sys.argv) > 1 else None))
