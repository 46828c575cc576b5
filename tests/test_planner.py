"""The library's kernel choice (qtts_w8a16_plan, host-only) on the talker and code-predictor shapes.

Pins the rule the B200 measurements chose: up to 16 rows the split-K streaming
kernel with the most CTAs holding a slice of K among the plans that run two per
SM (ties to the larger row tile; plans of 64- or 128-row tiles with at least two stages per
CTA first while they keep 128 CTAs with work), or at 9..16 rows the tcgen05 kernel where those CTAs
would stream >= 96 KiB each; up to 4 rows of int8 the whole-K
streaming kernel where it reaches more CTAs; past 16 rows the tcgen05 kernel, whose
batch tile grows to 128 columns past 64 rows only when 64-column tiles would not fit
one CTA per SM.
"""

from __future__ import annotations

import pytest

from qtts_b200 import _native as nat


@pytest.fixture(scope="module", autouse=True)
def _lib():
    nat.lib()  # raises if the library cannot be built or loaded


@pytest.mark.parametrize(
    "n,k,m,kernel,split,rows,ctas",
    [
        (4096, 2048, 1, "skinny_w8a16_kernel", 8, 128, 256),  # talker qkv
        (4096, 2048, 16, "skinny_w8a16_kernel", 8, 128, 256),
        # o_proj: 128 CTAs of 128 rows x 2 stages beat 256 one-stage CTAs
        (2048, 2048, 8, "skinny_w8a16_kernel", 8, 128, 128),
        (4096, 1024, 8, "skinny_w8a16_kernel", 4, 128, 128),  # code-predictor qkv
        # up to 4 rows the whole-K kernel only where the split-K plan loads some SMs twice:
        # not for code-predictor qkv (128 CTAs), still for talker gate_up (192)
        (4096, 1024, 1, "skinny_w8a16_kernel", 4, 128, 128),
        (12288, 2048, 2, "stream_w8a16_kernel", 1, 48, 256),
        (12288, 2048, 1, "stream_w8a16_kernel", 1, 48, 256),  # gate_up, few rows
        (12288, 2048, 8, "skinny_w8a16_kernel", 2, 128, 192),
        # 9..16 rows: tcgen05 where the split-K CTAs would stream >= 96 KiB each
        (12288, 2048, 16, "umma_w8a16_kernel", 1, 128, 96),
        (12288, 2048, 9, "umma_w8a16_kernel", 1, 128, 96),
        (2048, 6144, 16, "skinny_w8a16_kernel", 8, 64, 256),
        (2048, 6144, 4, "skinny_w8a16_kernel", 8, 64, 256),  # down_proj
        (4096, 2048, 32, "umma_w8a16_kernel", 4, 128, 128),
        (12288, 2048, 64, "umma_w8a16_kernel", 1, 128, 96),
        # code predictor o_proj / down_proj: 8 weight tiles, clusters of 8 (64 CTAs)
        (1024, 2048, 64, "umma_w8a16_kernel", 8, 128, 64),
        (1024, 3072, 32, "umma_w8a16_kernel", 8, 128, 64),
        (2048, 2048, 64, "umma_w8a16_kernel", 4, 128, 64),
        # past 64 rows: one 128-column tile when 64-column tiles would overflow a wave
        (12288, 2048, 128, "umma_w8a16_kernel", 1, 128, 96),
        (4096, 1024, 128, "umma_w8a16_kernel", 2, 128, 128),
        # code predictor down: 8 splits of 512 k, the last two without K (192 of 256 CTAs with
        # work) beat every plan whose CTAs all hold K (128 CTAs)
        (1024, 3072, 8, "skinny_w8a16_kernel", 8, 32, 256),
        (1024, 3072, 1, "skinny_w8a16_kernel", 8, 32, 256),
    ],
)
def test_auto_plans(n, k, m, kernel, split, rows, ctas):
    assert nat.plan(m, n, k) == {"kernel": kernel, "split": split, "row_tile": rows, "ctas": ctas}


def test_grouped_heads_and_forced_variants():
    assert nat.plan(8, 2048, 1024, groups=15) == {"kernel": "skinny_w8a16_kernel", "split": 1, "row_tile": 128,
                                                  "ctas": 240}
    assert nat.plan(8, 2048, 2048, variant=nat.variant_skinny(2, 4))["ctas"] == 32 * 2
    assert nat.plan(40, 2048, 2048, variant=nat.variant_umma(2))["split"] == 2
    assert nat.plan(2, 12288, 2048, variant=nat.variant_stream(6))["ctas"] == 128
    assert nat.plan(3, 80, 272, variant=nat.VARIANT_GENERIC)["kernel"] == "generic_w8a16_kernel"
    with pytest.raises(RuntimeError):
        nat.plan(32, 2048, 2048, variant=nat.variant_stream(0))  # the whole-K kernel takes M <= 16
    with pytest.raises(RuntimeError):
        nat.plan(1, 2048, 100)  # K % 16 != 0


def test_splits_give_most_ctas_work():
    """Slices are whole stages, so a split may leave its last CTAs without K; the planner
    keeps that to at most a quarter of a cluster on the talker and code-predictor shapes."""
    for n, k in [(1024, 3072), (2048, 6144), (4096, 2048), (6144, 1024), (3072, 2048), (80, 272)]:
        for m in (1, 2, 4, 8, 9, 16):
            p = nat.plan(m, n, k)
            if p["kernel"] == "skinny_w8a16_kernel" and p["split"] > 1:
                sw = 128 * (128 // p["row_tile"])  # k per stage: 8 warps / (row tile / 16) k groups
                kpc = -(-(-(-k // p["split"])) // sw) * sw
                with_k = min(p["split"], -(-k // kpc))
                assert 4 * with_k >= 3 * p["split"], (n, k, m, p)


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 17, 64])
def test_prologue_fuses_where_the_kernel_stages_activations(m):
    """RMSNorm / SiLU·up run inside the GEMM exactly when the chosen kernel is one of the
    two streaming kernels (int8, up to 16 rows, not where 9..16 rows go to the tcgen05
    kernel); otherwise the prologue kernel is chained."""
    lib = nat.lib()
    for n, k in ((4096, 2048), (12288, 2048), (2048, 6144), (3072, 1024)):
        for pro in (nat.PROLOGUE_RMSNORM, nat.PROLOGUE_SILU_MUL):
            fused = lib.qtts_w8a16_gemm_prologue_fused(m, n, k, pro, nat.VARIANT_AUTO)
            kernel = nat.plan(m, n, k)["kernel"]
            assert fused == (kernel in ("skinny_w8a16_kernel", "stream_w8a16_kernel")), (n, k, m)
            if m <= 8 or m > 16:
                assert fused == (m <= 8)
    assert lib.qtts_w8a16_gemm_prologue_fused(8, 4096, 2048, nat.PROLOGUE_RMSNORM, nat.variant_umma(1)) == 0
    assert lib.qtts_w8a16_gemm_prologue_fused(8, 4096, 2048, nat.PROLOGUE_RMSNORM, nat.variant_skinny(2)) == 1
    assert lib.qtts_w8a16_gemm_prologue_fused(8, 4096, 2048, 0, nat.VARIANT_AUTO) == 0
