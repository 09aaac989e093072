"""Weight pack codecs (numpy) — test infrastructure, see oracle/__init__.py.

Reference formats (byte-exact restatements):
  * fp16 crouton tile of W[K][N] (hexagon/mega/export_all.py:7-8 `wt16`): 32x32 tiles ordered
    [n block][k block]; inside a tile, halfword (k, n) sits at (k%32 // 2)*64 + (n%32)*2 + k%2.
  * q8 record (export_all_q8.py:10-18 `q8tiles`, Anima variant hexagon/mega/export_all.py:10-18):
    per tile s[c] = fp16(absmax_k |w[k][c]| / 127) with a floor (Anima: 0 -> 1.0; MOSS:
    < 6.2e-5 -> 6.2e-5), q = clip(rint(w/s), -127, 127), record = 64 halfwords of scales
    (halfword l = s[l//2]) + 1024 bytes u = q + 128 in tile order. Decoding
    (mkblk_test.py:23-27 `unpack`) gives q*s in fp32.
  * q4a record (moss/export_te.py:1-3, 21-40): 128 B scale vector, 128 B min vector, 512 B of
    nibbles (byte b of vector m: low nibble = halfword 256m+b, high = 256m+128+b); value = nib*s + m.

Device layouts (this runtime's own, hexanima_b200/csrc/gemm.cu header): W[N][K] row-major,
scale[K/group][N]; q4 nibbles packed 8 per 32-bit word with k at nibble (k>>1) + 4*(k&1).
"""
import numpy as np

F16_FLOOR_ANIMA = "anima"  # zero scale -> 1.0   (hexagon/mega/export_all.py:13)
F16_FLOOR_MOSS = "moss"    # scale < 6.2e-5 -> 6.2e-5 (moss/export_all_q8.py:13)


# ---------------------------------------------------------------- fp16 tiles
def wt16(w):
    """W[K][N] (float) -> fp16 tiles [nb][kb][16][32][2]; element [nb][kb][p][c][j] = W[32kb+2p+j][32nb+c]."""
    K, N = w.shape
    assert K % 32 == 0 and N % 32 == 0
    t = np.asarray(w, np.float32).astype(np.float16).reshape(K // 32, 16, 2, N // 32, 32)
    return np.ascontiguousarray(np.transpose(t, (3, 0, 1, 4, 2)))


def unwt16(t):
    """Inverse of wt16: tiles [nb][kb][16][32][2] -> W[K][N] (same dtype)."""
    nb, kb = t.shape[:2]
    return np.ascontiguousarray(np.transpose(t, (1, 2, 4, 0, 3)).reshape(kb * 32, nb * 32))


# ---------------------------------------------------------------- q8 records
def q8tiles(t, floor=F16_FLOOR_MOSS):
    """fp16 tiles (wt16 output) -> q8 record bytes, [nb][kb] x 1152 B."""
    a = t.astype(np.float32)
    nb, kb = a.shape[:2]
    s = np.abs(a).max(axis=(2, 4)) / np.float32(127.0)  # [nb][kb][32]
    if floor == F16_FLOOR_ANIMA:
        s = np.where(s == 0, np.float32(1.0), s)
    else:
        s = np.where(s < 6.2e-5, np.float32(6.2e-5), s)
    s16 = s.astype(np.float16)
    sf = s16.astype(np.float32)
    q = np.clip(np.rint(a / sf[:, :, None, :, None]), -127, 127).astype(np.int16)
    u = (q + 128).astype(np.uint8).reshape(nb, kb, 1024)
    scale_vec = np.repeat(s16, 2, axis=2).view(np.uint8).reshape(nb, kb, 128)
    return np.ascontiguousarray(np.concatenate([scale_vec, u], axis=2)).tobytes()


def _records(b, nb, kb, size):
    r = np.frombuffer(b, dtype=np.uint8)
    assert r.size == nb * kb * size, (r.size, nb, kb, size)
    return r.reshape(nb, kb, size)


def q8_scales(b, nb, kb):
    """fp16 scales [nb][kb][32] of q8 records."""
    return _records(b, nb, kb, 1152)[:, :, :128].copy().view(np.float16)[:, :, 0::2]


def unpack_q8(b, nb, kb):
    """q8 records -> W[K][N] float32 = q * s (mkblk_test.py:23-27)."""
    rec = _records(b, nb, kb, 1152)
    sc = q8_scales(b, nb, kb).astype(np.float32)
    q = (rec[:, :, 128:].astype(np.int16) - 128).reshape(nb, kb, 16, 32, 2).astype(np.float32)
    v = q * sc[:, :, None, :, None]
    return unwt16(v)


def dequant_q8_f16(b, nb, kb):
    """The operand the GPU multiplies: fp16(q * s) (q*s is exact in fp32, one RNE rounding)."""
    return unpack_q8(b, nb, kb).astype(np.float16)


# ---------------------------------------------------------------- q4a records
def q4a_tiles(q, S, M):
    """q [out][in] nibbles, S, M [out][in/32] -> q4a record bytes [nb][kb] x 768 (export_te.py:21-32)."""
    out, inn = q.shape
    nb, kb = out // 32, inn // 32
    # tile element (r = k within group, c = out within block), halfword order [r/2][c][r&1]
    t = q.reshape(nb, 32, kb, 32).transpose(0, 2, 3, 1)                     # [nb][kb][r][c]
    hw = t.reshape(nb, kb, 16, 2, 32).transpose(0, 1, 2, 4, 3).reshape(nb, kb, 1024)
    pairs = hw.reshape(nb, kb, 4, 2, 128)
    nib = (pairs[:, :, :, 0] | (pairs[:, :, :, 1] << 4)).astype(np.uint8)   # [nb][kb][4][128]
    s = S.reshape(nb, 32, kb).transpose(0, 2, 1).astype(np.float16)
    m = M.reshape(nb, 32, kb).transpose(0, 2, 1).astype(np.float16)
    rec = np.concatenate([np.repeat(s, 2, axis=2).view(np.uint8).reshape(nb, kb, 128),
                          np.repeat(m, 2, axis=2).view(np.uint8).reshape(nb, kb, 128),
                          nib.reshape(nb, kb, 512)], axis=2)
    return np.ascontiguousarray(rec).tobytes()


def unpack_q4a(b, nb, kb):
    """q4a records -> W[K][N] float32 = nib*s + m in float32 (export_te.py:33-40)."""
    rec = _records(b, nb, kb, 768)
    s = rec[:, :, :128].copy().view(np.float16)[:, :, 0::2].astype(np.float32)
    m = rec[:, :, 128:256].copy().view(np.float16)[:, :, 0::2].astype(np.float32)
    nib = rec[:, :, 256:].reshape(nb, kb, 4, 128)
    v = np.empty((nb, kb, 4, 2, 128), np.float32)
    v[:, :, :, 0] = nib & 15
    v[:, :, :, 1] = nib >> 4
    v = v.reshape(nb, kb, 16, 32, 2) * s[:, :, None, :, None] + m[:, :, None, :, None]
    return unwt16(v)


# ---------------------------------------------------------------- device layouts
def quant_q8(w_nk, group=32, floor=F16_FLOOR_MOSS):
    """W[N][K] -> (u8 [N][K] offset binary, fp16 scale [K/group][N]) with the q8tiles rule per group."""
    N, K = w_nk.shape
    a = np.asarray(w_nk, np.float32).astype(np.float16).astype(np.float32).reshape(N, K // group, group)
    s = np.abs(a).max(axis=2) / np.float32(127.0)
    if floor == F16_FLOOR_ANIMA:
        s = np.where(s == 0, np.float32(1.0), s)
    else:
        s = np.where(s < 6.2e-5, np.float32(6.2e-5), s)
    s16 = s.astype(np.float16)
    q = np.clip(np.rint(a / s16.astype(np.float32)[:, :, None]), -127, 127).astype(np.int16)
    u = (q + 128).astype(np.uint8).reshape(N, K)
    return np.ascontiguousarray(u), np.ascontiguousarray(s16.T)


def dequant_q8(u, scale, group):
    """Device q8 -> fp16 W[N][K] = fp16(q * s)."""
    N, K = u.shape
    q = u.astype(np.float32) - 128.0
    s = np.repeat(scale.T.astype(np.float32), group, axis=1)
    return (q * s).astype(np.float16)


def pack_nibbles(nib):
    """nib [N][K] values 0..15 -> u8 [N][K/2]; within each 32-bit word of 8 consecutive k, k sits at nibble (k>>1)+4(k&1)."""
    N, K = nib.shape
    g = nib.reshape(N, K // 8, 8).astype(np.uint32)
    pos = np.array([(k >> 1) + 4 * (k & 1) for k in range(8)], np.uint32)
    words = (g << (4 * pos)).sum(axis=2).astype(np.uint32)
    return np.ascontiguousarray(words.astype("<u4").view(np.uint8).reshape(N, K // 2))


def unpack_nibbles(packed):
    N, K2 = packed.shape
    words = np.ascontiguousarray(packed).view("<u4").reshape(N, K2 // 4).astype(np.uint32)
    pos = np.array([(k >> 1) + 4 * (k & 1) for k in range(8)], np.uint32)
    nib = (words[:, :, None] >> (4 * pos)) & 15
    return nib.reshape(N, K2 * 2).astype(np.uint8)


def quant_q4(w_nk, group=32):
    """Symmetric int4: s = fp16(absmax/7) (floored at 6.2e-5), q = clip(rint(w/s), -8, 7), nib = q + 8."""
    N, K = w_nk.shape
    a = np.asarray(w_nk, np.float32).astype(np.float16).astype(np.float32).reshape(N, K // group, group)
    s = np.abs(a).max(axis=2) / np.float32(7.0)
    s = np.where(s < 6.2e-5, np.float32(6.2e-5), s)
    s16 = s.astype(np.float16)
    q = np.clip(np.rint(a / s16.astype(np.float32)[:, :, None]), -8, 7).astype(np.int16)
    nib = (q + 8).astype(np.uint8).reshape(N, K)
    return pack_nibbles(nib), np.ascontiguousarray(s16.T)


def dequant_q4(packed, scale, group=32):
    nib = unpack_nibbles(packed).astype(np.float32) - 8.0
    s = np.repeat(scale.T.astype(np.float32), group, axis=1)
    return (nib * s).astype(np.float16)


def quant_q4a(w_nk, group=32):
    """Asymmetric int4 (q4a): m = fp16(min), s = fp16((max-min)/15), nib = clip(rint((w-m)/s), 0, 15)."""
    N, K = w_nk.shape
    a = np.asarray(w_nk, np.float32).reshape(N, K // group, group)
    lo, hi = a.min(axis=2), a.max(axis=2)
    s = np.maximum((hi - lo) / np.float32(15.0), np.float32(6.2e-5)).astype(np.float16)
    m = lo.astype(np.float16)
    nib = np.clip(np.rint((a - m.astype(np.float32)[:, :, None]) / s.astype(np.float32)[:, :, None]), 0, 15)
    nib = nib.astype(np.uint8).reshape(N, K)
    return pack_nibbles(nib), np.ascontiguousarray(s.T), np.ascontiguousarray(m.T)


def dequant_q4a(packed, scale, minv, group=32):
    """fp16(fp32(nib*s) + m): the float32 multiply-then-add of unpack_q4a, rounded once to fp16."""
    nib = unpack_nibbles(packed).astype(np.float32)
    s = np.repeat(scale.T.astype(np.float32), group, axis=1)
    m = np.repeat(minv.T.astype(np.float32), group, axis=1)
    return ((nib * s).astype(np.float32) + m).astype(np.float16)


def q8_records_to_device(b, nb, kb):
    """q8 records -> device (u8 [N][K], fp16 scale [K/32][N]): what the GPU repack produces."""
    rec = _records(b, nb, kb, 1152)
    u = rec[:, :, 128:].reshape(nb, kb, 16, 32, 2)
    w = unwt16(u)                        # [K][N] u8
    sc = q8_scales(b, nb, kb)            # [nb][kb][32]
    scale = np.ascontiguousarray(sc.transpose(1, 0, 2).reshape(kb, nb * 32))
    return np.ascontiguousarray(w.T), scale


def situ_rows(up_nk, gate_nk):
    """MOSS up/gate [F][K] each -> device up_gate [2F][K]: per 256 rows, 128 up then the 128 matching gate rows."""
    F, K = up_nk.shape
    assert F % 128 == 0
    u = up_nk.reshape(F // 128, 128, K)
    g = gate_nk.reshape(F // 128, 128, K)
    return np.ascontiguousarray(np.concatenate([u, g], axis=1).reshape(2 * F, K))


def interleave32(up_kn, gate_kn):
    """Pack column order of MOSS up_gate (export_moss.py:17-19): 32-column blocks (up_j, gate_j)."""
    K, F = up_kn.shape
    return np.stack((up_kn.reshape(K, F // 32, 32), gate_kn.reshape(K, F // 32, 32)), 2).reshape(K, 2 * F)


# ---------------------------------------------------------------- LoRA fold into q8 base tiles
def lora_fold_q8(u, scale, group, B, A, lscale=1.0, floor=F16_FLOOR_MOSS, k_base=None):
    """Device q8 (u8 [N][K], fp16 scale [K/group][N]) with lscale * B[N][r] @ A[r][k_base] added to
    columns [0, k_base), each group requantised with the quant_q8 rule (the rule of the reference's fold
    tool, moss/mossrun/lorafold.cpp:138-156). B rows are in device row order.

    The arithmetic order is part of the definition (the device kernel follows it): the rank sum runs
    r = 0, 1, ... with each product and each sum rounded to float32, then v = q*s + fl(lscale * sum)."""
    N, K = u.shape
    kb = K if k_base is None else k_base
    B = np.asarray(B, np.float32)
    A = np.asarray(A, np.float32)
    acc = np.zeros((N, kb), np.float32)
    for r in range(B.shape[1]):
        acc = acc + np.outer(B[:, r], A[r])
    sc = np.repeat(scale[:kb // group].T.astype(np.float32), group, axis=1)
    v = (u[:, :kb].astype(np.float32) - np.float32(128)) * sc + np.float32(lscale) * acc
    nu, ns = quant_q8(v, group, floor)
    out_u, out_s = u.copy(), scale.copy()
    out_u[:, :kb] = nu
    out_s[:kb // group] = ns
    return out_u, out_s


def fold_slots(BT, AM, keep=128):
    """The rank-128 LoRA slot fold of the reference's fold tool (moss/mossrun/lorafold.cpp:200-284
    `fold`), restated in numpy float64: BT [R][N] (turbo B^T rows then scaled user B^T rows), AM [R][I]
    (turbo A rows then user A rows). Returns float32 B' [keep][N], A' [keep][I] with B'^T A' the best
    rank-`keep` approximation of BT^T AM, singular values on the B side:
      Gb = BT BT^T = Vb diag(lb) Vb^T, Ga = AM AM^T = Va diag(la) Va^T (eigenvalues below 1e-12 of the
      largest dropped), core C = Sb Vb^T Va Sa = U S W^T, B' = S_k U_k^T Sb^-1 Vb^T BT,
      A' = W_k^T Sa^-1 Va^T AM."""
    BT = np.asarray(BT, np.float64)
    AM = np.asarray(AM, np.float64)
    lb, Vb = np.linalg.eigh(BT @ BT.T)
    la, Va = np.linalg.eigh(AM @ AM.T)

    def roots(lam):
        ok = lam > lam.max() * 1e-12
        sq = np.where(ok, np.sqrt(np.where(ok, lam, 1.0)), 0.0)
        return sq, np.where(ok, 1.0 / np.where(ok, sq, 1.0), 0.0)

    sb, ib = roots(lb)
    sa, ia = roots(la)
    C = (sb[:, None] * (Vb.T @ Va)) * sa[None, :]
    U, S, Wt = np.linalg.svd(C)
    k = min(keep, len(S))
    S = np.where(S[:k] > S[0] * 1e-12, S[:k], 0.0)
    Tb = (Vb * ib[None, :]) @ (U[:, :k] * S[None, :])      # [R][k]
    Ta = Wt[:k] @ (ia[:, None] * Va.T)                      # [k][R]
    Bo = np.zeros((keep, BT.shape[1]))
    Ao = np.zeros((keep, AM.shape[1]))
    Bo[:k] = Tb.T @ BT
    Ao[:k] = Ta @ AM
    return Bo.astype(np.float32), Ao.astype(np.float32)


def situ_logical_rows(n_rows):
    """Device row r of a MOSS up_gate matrix -> its logical row ([0,F) up, [F,2F) gate); inverse view of situ_rows."""
    F = n_rows // 2
    r = np.arange(n_rows)
    o = (r // 256) * 128 + (r % 256) % 128
    return np.where(r % 256 < 128, o, F + o)
