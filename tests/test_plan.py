"""Kernel choices of hx_gemm / hx_attention, answered on the host (hx_gemm_query / hx_attention_query)
without a GPU, at the Anima block's shapes on a 148-SM B200: which GEMM kernel runs (single-CTA tiles,
CTA pairs, q8 weights in TMEM), when quantised weights are expanded to fp16 first, when the CTA pairs
take 224-column tiles or a stream-K tail, and when the short-key attention kernel is taken."""
import pytest

from hexanima_b200 import build, runtime as rt

SM = 148
D, F, CD, T, C = 2048, 8192, 1024, 1536, 256
SINGLE, PAIR, TMEM_W = 1, 2, 3


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def q(m, n, k, epi, fmt=rt.FMT_Q8, group=64, **kw):
    return rt.gemm_query(m, n, k, fmt, epi, group=group, sm_count=SM, **kw)


def test_one_image_projections():
    M = T
    qkv = q(M, 3 * D, D, rt.EPI_RMS)      # 144 TMEM-weight tiles fill the 74 pairs
    assert (qkv["kernel"], qkv["expand"], qkv["tiles"]) == (TMEM_W, 0, 144)
    o = q(M, D, D, rt.EPI_RESID)          # one wave (48 tiles), short K: no stream-K
    assert (o["kernel"], o["streamk"], o["tiles"]) == (TMEM_W, 0, 48)
    cq = q(M, D, D, rt.EPI_RMS)
    assert cq["kernel"] == TMEM_W
    ckv = q(C, 2 * D, CD, rt.EPI_RMS)     # the per-sample cross-attention k|v
    assert ckv["kernel"] == TMEM_W


def test_one_image_mlp():
    m1 = q(T, F, D, rt.EPI_GELU)          # 37 tiles of 224 per band: 222 = 3 waves on 74 pairs
    assert (m1["kernel"], m1["expand"], m1["tile_n"], m1["tiles"]) == (PAIR, 0, 224, 222)
    m2 = q(T, D, F, rt.EPI_RESID)         # 48 pair tiles of 128 k-blocks: stream-K tail
    assert (m2["kernel"], m2["streamk"], m2["tile_n"]) == (PAIR, 1, 256)


def test_two_images_expand_then_fp16_pairs():
    M = 2 * T
    m1 = q(M, F, D, rt.EPI_GELU)
    assert (m1["expand"], m1["kernel"], m1["tile_n"], m1["tiles"]) == (1, PAIR, 224, 444)
    qkv = q(M, 3 * D, D, rt.EPI_RMS)      # fp16 weights: the CTA-pair kernel with whole heads per tile
    assert (qkv["expand"], qkv["kernel"], qkv["tile_n"]) == (1, PAIR, 256)
    m2 = q(M, D, F, rt.EPI_RESID)         # 96 pair tiles: the last 22 cut into stream-K shares
    assert (m2["expand"], m2["kernel"], m2["streamk"]) == (1, PAIR, 1)
    below = q(M - 1, F, D, rt.EPI_GELU)   # the expansion starts at 3072 rows
    assert below["expand"] == 0


@pytest.mark.parametrize("images,tile_n", [(4, 256), (8, 256)])
def test_four_and_eight_images_keep_256_columns(images, tile_n):
    m1 = q(images * T, F, D, rt.EPI_GELU)  # 224 would need more waves (12 against 11 at four images)
    assert (m1["expand"], m1["kernel"], m1["tile_n"], m1["streamk"]) == (1, PAIR, tile_n, 0)


def test_forced_tiles_and_rejections():
    assert q(T, F, D, rt.EPI_GELU, tile=1)["kernel"] == SINGLE
    assert q(T, F, D, rt.EPI_GELU, tile=2)["tile_n"] == 224  # pairs, the wave rule still picks 224
    assert q(T, F, D, rt.EPI_STORE, tile=5)["tile_n"] == 224
    assert q(T, F, D, rt.EPI_GELU, tile=4)["expand"] == 1
    with pytest.raises(rt.HxError):
        q(T, D, D, rt.EPI_RESID, tile=5)                     # 224 columns: GELU / store epilogues only
    with pytest.raises(rt.HxError):
        q(T, F, D, rt.EPI_GELU, fmt=rt.FMT_Q4, group=32, tile=5)
    with pytest.raises(rt.HxError):
        q(T, F, D, rt.EPI_GELU, fmt=rt.FMT_F16, tile=3)    # the TMEM-weight kernel takes q8 weights
    with pytest.raises(rt.HxError):
        q(T, F, D - 32, rt.EPI_GELU)                         # K not a multiple of 64


@pytest.mark.parametrize("batch,kernel", [(1, 2), (2, 2), (4, 2), (8, 1)])
def test_cross_attention_kernel_by_batch(batch, kernel):
    # 12 query tiles x 16 heads per image: short-key kernel up to six tiles per SM (888 tiles)
    assert rt.attention_query(batch, 16, T, C, sm_count=SM) == kernel


def test_attention_routing_rules():
    assert rt.attention_query(1, 16, T, T, sm_count=SM) == 1          # self-attention: general kernel
    assert rt.attention_query(1, 16, T, 128, sm_count=SM) == 1        # one key tile: general kernel
    assert rt.attention_query(1, 16, T, 100, kernel=2, sm_count=SM) == 2
    assert rt.attention_query(8, 16, T, C, kernel=2, sm_count=SM) == 2
    assert rt.attention_query(1, 16, T, C, sm_count=SM, o_addr=(1 << 20) + 8) == 1  # TMA stores need 16 B
    with pytest.raises(rt.HxError):
        rt.attention_query(1, 16, T, 300, kernel=2, sm_count=SM)
    with pytest.raises(rt.HxError):
        rt.attention_query(1, 16, T, C, kernel=3, sm_count=SM)


def test_moss_shapes():
    """MOSS 1 Mpx block (q4 g32, hidden 3072, MLP 12288, SiTU): 4608 tokens on one GPU expand to fp16; a
    rank of the 8-way Ulysses split (576 tokens) dequantises in the main loop."""
    MD, MF = 3072, 12288
    full = rt.gemm_query(4608, 2 * MF, MD, rt.FMT_Q4, rt.EPI_SITU, group=32, sm_count=SM)
    assert (full["expand"], full["kernel"], full["tile_n"]) == (1, PAIR, 256)
    rank8 = rt.gemm_query(576, 2 * MF, MD, rt.FMT_Q4, rt.EPI_SITU, group=32, sm_count=SM)
    assert (rank8["expand"], rank8["kernel"]) == (0, PAIR)
    qkv8 = rt.gemm_query(576, 3 * MD, MD, rt.FMT_Q4, rt.EPI_RMS, group=32, sm_count=SM)
    assert qkv8["expand"] == 0 and qkv8["kernel"] in (SINGLE, PAIR)  # the TMEM-weight kernel takes q8 only
    # the joint attention over the whole sequence on 3 of the 24 heads: general kernel
    assert rt.attention_query(1, 3, 4608, 4608, sm_count=SM) == 1
