"""Host-side invariants of the decode GEMV's launch plan (plan_gemv, csrc/gemv.cu).

No GPU: a small C++ program links the in-tree libq35k.so, asks for the plan of
many shapes and prints it; the test checks what the kernels rely on (grid,
split-K clusters, the register-budget variants, shared memory).
"""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "qwen3.5sharp_b200", "csrc")
LIB_DIR = os.path.join(ROOT, "qwen3.5sharp_b200")
CUDA_INC = "/usr/local/cuda/include"

HARNESS = r"""
#include "kernels.h"
#include <cstdio>
int main() {
    const int types[3] = {12, 13, 14};
    const int nbs[] = {1, 2, 3, 4, 8, 10, 11, 14, 16, 17, 20, 21, 38, 40, 64};
    const int ns[] = {1, 32, 33, 64, 608, 2560, 4736, 4753, 9728, 19456, 27648, 151936};
    for (int t : types)
        for (int nb : nbs)
            for (int n : ns)
                for (int m = 1; m <= 8; m++) {
                    q35k::GemvPlan p = q35k::plan_gemv(t, nb, n, m, 148);
                    std::printf("%d %d %d %d %d %d %d %d %d %d %d %zu %d %d\n", t, nb, n, m, p.groups, p.grid,
                                p.splits, p.unit_blocks, p.warps, p.threads, p.cluster, p.smem_bytes, (int)p.fits,
                                (int)p.three_per_sm);
                }
}
"""


@pytest.fixture(scope="module")
def plans(tmp_path_factory):
    lib = os.path.join(LIB_DIR, "libq35k.so")
    cxx = shutil.which("g++")
    if not (os.path.exists(lib) and cxx and os.path.exists(os.path.join(CUDA_INC, "cuda_runtime.h"))):
        pytest.skip("needs the built libq35k.so, g++ and the CUDA headers")
    d = tmp_path_factory.mktemp("plan")
    src, exe = os.path.join(d, "plan.cpp"), os.path.join(d, "plan")
    with open(src, "w") as f:
        f.write(HARNESS)
    subprocess.run([cxx, "-std=c++17", "-I", CSRC, "-I", CUDA_INC, src, "-o", exe, "-L", LIB_DIR, "-lq35k",
                    f"-Wl,-rpath,{LIB_DIR}"], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    rows = []
    for line in out.splitlines():
        v = line.split()
        rows.append(dict(zip(("type", "nb", "n", "m", "groups", "grid", "splits", "u", "warps", "threads",
                              "cluster", "smem", "fits", "three"), [int(x) for x in v])))
    return rows


def test_plan_covers_every_row_and_block(plans):
    for p in plans:
        assert p["groups"] == (p["n"] + 31) // 32
        assert p["grid"] == p["groups"] * p["splits"]
        assert p["splits"] == -(-p["nb"] // p["u"]), p
        assert 1 <= p["warps"] <= 20 and p["threads"] == 32 * p["warps"]
        assert p["fits"] == 1 and p["smem"] <= 227 * 1024


def test_split_k_clusters(plans):
    """2..8 K-splits form one portable cluster (grid a multiple of it); more
    splits, or none, use no cluster."""
    for p in plans:
        if 2 <= p["splits"] <= 8:
            assert p["cluster"] == p["splits"] and p["grid"] % p["cluster"] == 0, p
        else:
            assert p["cluster"] == 0, p


def test_register_budget_variant(plans):
    """The three-CTAs-per-SM kernel (320 threads at most) only for one or two
    tokens, and only where three such CTAs per SM hold the grid or the shared
    memory allows no more."""
    for p in plans:
        if p["three"]:
            assert p["m"] <= 2 and p["warps"] <= 10, p
            smem_fit = 233472 // (p["smem"] + 1024)
            assert smem_fit <= 3 or p["grid"] <= 3 * 148, p


def test_mma_token_counts_use_at_most_ten_warps(plans):
    for p in plans:
        mma_min = 6 if p["type"] == 14 else 3
        if p["m"] >= mma_min or p["splits"] > 1:
            assert p["warps"] <= 10, p
