"""Kernel selection and launch planning on the host (w4a16_plan_shape), without a GPU.

The expected choices are the ones measured fastest on B200 for the merged Llama-2-7B
decoder layer (qkv 4096->12288, o 4096->4096, gate_up 4096->22016, down 11008->4096),
and the invariants are the planners' own rules.
"""
import itertools

import pytest
import torch

from drofell_for_revision_b200 import _capi

SMS = 148
LAYER = {"qkv": (4096, 12288), "o": (4096, 4096), "gate_up": (4096, 22016), "down": (11008, 4096)}
GEMV, EXACT, GEMV_MMA = _capi.KERN_GEMV, _capi.KERN_EXACT, _capi.KERN_GEMV_MMA


def plan(K, N, M, g=128, path=_capi.PATH_AUTO, dtype=torch.float16, act=False):
    return _capi.plan_shape(K, N, K // g if g > 0 else 1, M, dtype, path, SMS, act_order=act)


@pytest.mark.parametrize("name,wide,splits", [("qkv", True, 4), ("o", False, 8), ("gate_up", True, 2),
                                              ("down", False, 8)])
def test_decode_m1_layer_plans(name, wide, splits):
    K, N = LAYER[name]
    (kern, tile, sp, rows), is_wide, ws = plan(K, N, 1)
    assert (kern, tile, rows) == (GEMV, 128, 1)
    assert is_wide == wide  # WIDE (3 CTAs per SM) only on the wide, short-K shapes
    assert sp == splits
    assert ws == 0


@pytest.mark.parametrize("M", [8, 16])
@pytest.mark.parametrize("name", sorted(LAYER))
def test_decode_batch_layer_is_one_pass_on_mma(name, M):
    K, N = LAYER[name]
    (kern, tile, sp, rows), _, ws = plan(K, N, M)
    # all M rows of X in one pass over the weight; a CTA covers 1, 2 or 4 stripes of 64
    # columns and a cluster of up to 16 CTAs splits K
    assert kern == GEMV_MMA and tile in (64, 128, 256) and rows == M
    assert 1 <= sp <= 16 and ws == 0


@pytest.mark.parametrize("name", sorted(LAYER))
def test_prefill_full_shapes_do_not_split(name):
    K, N = LAYER[name]
    (kern, tile, sp, cps), _, ws = plan(K, N, 2048)
    assert (kern, tile, sp) == (EXACT, 256, 1)
    assert cps == K // 64 and ws == 0


@pytest.mark.parametrize("K,N", [(4096, 1024), (11008, 1024), (4096, 512), (11008, 512), (4096, 1536)])
def test_prefill_narrow_shards_split_k_with_partials(K, N):
    M = 2048
    (kern, tile, sp, cps), _, ws = plan(K, N, M)
    assert kern == EXACT and tile == 256
    assert sp > 1 and (sp - 1) * cps < K // 64 <= sp * cps  # no empty split
    assert ws == sp * M * N * 4  # fp32 partials, summed by the reduce kernel


def test_act_order_adds_the_x_gather_to_the_workspace():
    for M in (1, 8, 300):
        _, _, ws_plain = plan(4096, 4096, M)
        _, _, ws_act = plan(4096, 4096, M, act=True)
        assert ws_act - ws_plain == (M * 4096 * 2 + 255) // 256 * 256


def test_cuda_core_gemv_never_fills_a_single_wave(monkeypatch):
    """A single wave over 90 % of the CTA slots leaves the next kernel no room to start
    early under PDL (measured up to 27 % slower), so the planner never picks one. (Planned
    for a handle without the repacked copy: the CUDA-core kernel at every shape.)"""
    monkeypatch.setenv("W4A16_NO_REPACK", "1")
    for K, N in itertools.product([1024, 2048, 4096, 8192, 11008, 14336, 28672],
                                  [1024, 2048, 4096, 5504, 8192, 11008, 12288, 14336, 22016, 28672, 57344]):
        (kern, tile, sp, rows), wide, _ = plan(K, N, 1, path=_capi.PATH_GEMV)
        assert kern == GEMV and 1 <= sp <= 8
        slots = (3 if wide else 2) * SMS
        ctas = (N + tile - 1) // tile * sp
        assert not (slots * 0.9 < ctas <= slots), (K, N, sp, wide)


def test_path_choices():
    K, N = 4096, 4096
    for dt in (torch.float16, torch.bfloat16):
        assert plan(K, N, 1, path=_capi.PATH_TC, dtype=dt)[0][0] == EXACT  # PATH_TC is the exact-W GEMM at any M
    assert plan(K, N, 16, path=_capi.PATH_TC_EXACT)[0][0] == EXACT
    assert plan(K, N, 17)[0][0] == EXACT
    for M in (1, 2):
        assert plan(K, N, M)[0][0] == GEMV
    for M in (3, 8, 16):
        assert plan(K, N, M)[0][0] == GEMV_MMA


def test_shape_errors():
    with pytest.raises(_capi.W4A16Error) as e:
        _capi.plan_shape(4096, 100, 32, 1)  # N not a multiple of 32
    assert e.value.code == _capi.W4A16_ERR_INVALID
    with pytest.raises(_capi.W4A16Error) as e:
        _capi.plan_shape(4096, 4096, 4096 // 12, 1)  # does not divide K
    assert e.value.code == _capi.W4A16_ERR_INVALID
    with pytest.raises(_capi.W4A16Error) as e:
        _capi.plan_shape(192, 64, 48, 1)  # group size 4
    assert e.value.code == _capi.W4A16_ERR_UNSUPPORTED


@pytest.mark.parametrize("M", [32, 128, 256])
def test_mid_m_70b_projections_run_in_the_natural_orientation(M):
    # a tcgen05 MMA costs about the same for any N on B200: with 128 tokens or fewer the
    # weight goes on the N side (256 columns per instruction)
    for K, N in [(8192, 28672), (8192, 57344), (28672, 8192)]:
        assert _capi.plan_orientation(K, N, K // 128, M) == "natural", (K, N, M)


def test_prefill_runs_swap_ab_and_decode_is_a_gemv():
    assert _capi.plan_orientation(4096, 11008, 32, 2048) == "swap"
    assert _capi.plan_orientation(4096, 11008, 32, 8) == ""


def test_long_k_16_rows_take_the_gemm_instead_of_two_gemv_passes():
    (kern, _, _, rows), _, _ = plan(28672, 8192, 16)
    assert kern == EXACT and _capi.plan_orientation(28672, 8192, 224, 16) == "natural"
    (kern, _, _, rows), _, _ = plan(28672, 8192, 8)
    assert kern == GEMV_MMA and rows == 8


SHARDED_LAYERS = {"7b": [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)],
                  "70b": [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]}


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("model", sorted(SHARDED_LAYERS))
def test_every_rank_shard_of_the_sharded_runs_has_a_plan(model, P):
    # the shapes each rank of `bench.py --gpus P` runs, at every M the bench times there
    for K, N in SHARDED_LAYERS[model]:
        n = N // P
        assert N % P == 0 and n % 8 == 0  # qzeros packs 8 columns per word
        for M in (1, 8, 16, 128, 2048):
            (kern, tile, sp, per), _, ws = plan(K, n, M)
            assert kern in (GEMV, GEMV_MMA, EXACT)
            assert tile in (64, 128, 256) and sp >= 1 and per >= 1
            if kern == EXACT:
                assert (sp - 1) * per < K // 64 <= sp * per  # every K chunk once, no empty split
                assert ws == (0 if sp == 1 else sp * M * n * 4)
            else:
                assert ws == 0 and sp <= 16


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("K,N", SHARDED_LAYERS["70b"] + [(8192, 28672), (5120, 27648)])
def test_wide_long_k_decode_runs_the_mma_gemv(K, N, M):
    # K >= 8192 and N >= 8192, or K > 4096 and N >= 16384: the mma.sync GEMV streams these
    # faster than the CUDA-core kernel, whose WIDE configuration stops at K = 4096
    assert plan(K, N, M)[0][0] == GEMV_MMA


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("K,N", SHARDED_LAYERS["7b"] + [(5120, 15360), (13824, 5120), (8192, 7168), (8192, 1024)])
def test_other_decode_shapes_stay_on_cuda_cores(K, N, M):
    assert plan(K, N, M)[0][0] == GEMV
