"""The table read's shared-memory plan on the host (tests/plan_check.cu over mv_plan in common.cuh): for the Seoul
tables (Q4_0 and Q4_1 rows) at 1, 2, 4 and 8 inputs, every region is aligned, the regions follow one another without
overlap, the total fits one CTA's budget, weight stages hold their rows, and the decode plans (1 and 2 inputs) keep
full stages. The plans are the engine's own (mv_plan_stages)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
MV_NBUF, MV_MAX_STAGES, MV_STAGE_BYTES = 4, 8, 36864
MV_SMEM_BUDGET = 220 * 1024


@pytest.fixture(scope="module")
def plans(tmp_path_factory):
    if not (os.path.exists(NVCC) or shutil.which("nvcc")):
        pytest.skip("nvcc not found")
    exe = str(tmp_path_factory.mktemp("plan") / "plan_check")
    r = subprocess.run([NVCC if os.path.exists(NVCC) else "nvcc", "-std=c++17", "-x", "cu",
                        os.path.join(ROOT, "tests", "plan_check.cu"), "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.splitlines()
    rows = []
    for line in out:
        name, nc, *kv = line.split()
        d = {k: int(v) for k, v in (x.split("=") for x in kv)}
        d["name"] = name
        rows.append(d)
    return rows


def test_regions_aligned_ordered_and_within_budget(plans):
    assert len(plans) == 9 * 4
    for p in plans:
        nc, nb, sr, ns, hm = p["nc"], p["nb"], p["sr"], p["ns"], p["hm"]
        ld = nb + 4
        assert sr >= 1 and ns >= 1, p
        assert p["stage"] == 0 and p["sstride"] % 128 == 0 and sr * p["rb"] <= p["sstride"], p
        assert sr * p["rb"] <= MV_STAGE_BYTES, p
        assert p["bar"] >= ns * p["sstride"] and p["bar"] % 8 == 0, p
        for k in ("xq", "xd", "xs", "fs", "dd", "vo", "ab", "pc", "red", "total"):
            assert p[k] % 16 == 0, (k, p)
        assert p["xq"] >= p["bar"] + 8 * MV_MAX_STAGES
        assert p["xd"] >= p["xq"] + nc * 32 * nb
        assert p["xs"] >= p["xd"] + 4 * nc * nb and p["fs"] >= p["xs"] + 4 * nc * nb
        assert p["dd"] >= p["fs"] + MV_NBUF * 4 * nc * sr * ld
        assert p["vo"] >= p["dd"] + (2 if hm else 1) * MV_NBUF * 2 * sr * ld
        assert p["vb"] == p["fs"] and p["ab"] >= max(p["vo"], p["vb"] + 4 * nc * p["vb_len"])
        assert p["pc"] >= p["ab"] + 4 * nc * p["ab_len"] and p["red"] > p["pc"] and p["total"] > p["red"]
        assert p["total"] <= p["budget"], p


def test_decode_plans_keep_full_stages(plans):
    for p in plans:
        if p["nc"] <= 2:
            assert p["sr"] == p["full"], p
            if p["full"] * p["rb"] == MV_STAGE_BYTES:
                assert p["sstride"] == MV_STAGE_BYTES, p


def test_eight_inputs_keep_two_stages_in_flight(plans):
    for p in plans:
        if p["nc"] == 8 and p["rows_cta"] > p["sr"]:
            assert p["ns"] >= 2, p
