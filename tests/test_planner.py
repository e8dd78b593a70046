"""The launch planner on CPU, through b2g_plan_for_device (the plan b2g_create
makes, for a given SM count and shared-memory limit, without a device).

The decode shapes' plans are the ones the B200 runs use (the bench reports
gate||up on 128 whole-tile CTAs and down on 96); the rest pins the planner's
rules: whole tiles when K is whole and the largest share is at most 1.6x the
even share, K split only when max_m rows of x exceed 128 KB, and more CTAs
(run as waves) when one per SM would overflow a CTA's shared slots."""
from __future__ import annotations

import pytest

from conftest import load_b2g

UNITS, TILES = 1, 2


@pytest.fixture(scope="module")
def P():
    return load_b2g()


def plan(P, K, N, **kw):
    return P.plan_for_device(K, N, **kw)


@pytest.mark.parametrize("wd", ["fp8_e4m3", "fp16"])
def test_decode_mlp_shapes(P, wd):
    gu = plan(P, 3072, 8192, weight_dtype=wd, fuse=P.FUSE_GATE_UP_SILU | P.FUSE_RMSNORM_INPUT)
    assert (gu["grid"], gu["partition"], gu["ksplit"], gu["n_slots"], gu["max_contrib"]) == (128, TILES, 1, 4, 1)
    dn = plan(P, 8192, 3072, weight_dtype=wd, fuse=P.FUSE_RESIDUAL_ADD)
    assert (dn["grid"], dn["partition"], dn["ksplit"], dn["n_slots"], dn["max_contrib"]) == (96, TILES, 1, 2, 1)
    wb = 1 if wd == "fp8_e4m3" else 2
    assert gu["packed_bytes"] == 2 * 3072 * 8192 * wb and dn["packed_bytes"] == 8192 * 3072 * wb
    assert gu["smem_bytes"] <= P.B200_SMEM_OPTIN and dn["smem_bytes"] <= P.B200_SMEM_OPTIN


def test_tensor_parallel_shards(P):
    G = P.FUSE_GATE_UP_SILU | P.FUSE_RMSNORM_INPUT
    for tp, gu_grid in ((2, 128), (4, 128), (8, 64)):
        gu = plan(P, 3072, 8192 // tp, fuse=G)
        dn = plan(P, 8192 // tp, 3072)
        assert (gu["grid"], gu["partition"]) == (gu_grid, TILES), tp
        assert (dn["grid"], dn["partition"], dn["ksplit"]) == (96, TILES, 1), tp


def test_whole_tiles_rule(P):
    # 300 tiles: 3 per CTA on 100 CTAs against 2.03 on 148 (1.48x) -> whole tiles
    p = plan(P, 1024, 300 * 16)
    assert (p["grid"], p["partition"]) == (100, TILES)
    # 149 tiles: 2 per CTA against 1.007 (1.99x) -> split tiles on every SM
    p = plan(P, 1024, 149 * 16)
    assert (p["grid"], p["partition"]) == (148, UNITS) and p["max_contrib"] == 2
    # fewer tiles than SMs: one each
    p = plan(P, 1024, 64 * 16)
    assert (p["grid"], p["partition"]) == (64, TILES)


def test_k_split_rule(P):
    # max_m rows of x within 128 KB: K whole
    assert plan(P, 8192, 3072)["ksplit"] == 1
    assert plan(P, 16384, 3072, max_m=4)["ksplit"] == 1
    # beyond: the most ranges that keep >= 2048 k each
    p = plan(P, 16384, 3072)
    assert p["ksplit"] == 8 and p["partition"] == UNITS
    assert plan(P, 12288, 3072)["ksplit"] == 4
    # RMSNorm needs whole rows: never split; refused when they do not fit
    assert plan(P, 8192, 3072, fuse=P.FUSE_RMSNORM_INPUT)["ksplit"] == 1
    with pytest.raises(P.B2GError) as e:
        plan(P, 16384, 3072, fuse=P.FUSE_RMSNORM_INPUT)
    assert e.value.status == 5  # B2G_ERR_OOM: 8 rows x 16384 halves exceed shared memory


def test_wide_outputs_run_in_waves(P):
    p = plan(P, 3072, 128256)  # lm_head: 8016 tiles
    assert p["n_tiles"] == 8016 and p["n_slots"] <= 8 and p["partition"] == TILES
    assert p["grid"] > 148 and p["grid"] * p["n_slots"] >= p["n_tiles"]
    assert p["packed_bytes"] == 3072 * 128256
    # the same shape on a GPU with more SMs needs fewer waves, never more CTAs
    assert plan(P, 3072, 128256, num_sms=1024)["grid"] <= p["grid"]


def test_other_gpus_and_errors(P):
    assert plan(P, 3072, 8192, num_sms=132)["grid"] <= 132
    with pytest.raises(P.B2GError):
        plan(P, 3072, 8192, num_sms=0)
    with pytest.raises(P.B2GError):
        plan(P, 3072, 8192, max_m=9)
    with pytest.raises(P.B2GError):
        plan(P, 3072, 8192, m=9)
    with pytest.raises(P.B2GError):
        plan(P, 3072, 8192, smem_optin=4096)  # not even one CTA's x rows fit
