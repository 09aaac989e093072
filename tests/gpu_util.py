"""Helpers for the GPU tests: device weight sets built from oracle quantisers, comparisons."""
import numpy as np
import torch

from hexanima_b200 import runtime as rt
from oracle import packs as op

FMT_NAMES = {rt.FMT_F16: "f16", rt.FMT_Q8: "q8", rt.FMT_Q4: "q4", rt.FMT_Q4A: "q4a"}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_mat(fmt, w_nk, group=32):
    """w_nk float [N][K] -> (hx_mat, tensors to keep alive, operand values fp32 [N][K] on the CPU)."""
    w = np.asarray(w_nk, np.float32)
    N, K = w.shape
    if fmt == rt.FMT_F16:
        w16 = w.astype(np.float16)
        t = dev(w16)
        return rt.make_mat(fmt, N, K, t, group=64), [t], torch.from_numpy(w16.astype(np.float32))
    if fmt == rt.FMT_Q8:
        u, s = op.quant_q8(w, group)
        tu, ts = dev(u), dev(s)
        deq = op.dequant_q8(u, s, group)
        return rt.make_mat(fmt, N, K, tu, ts, group=group), [tu, ts], torch.from_numpy(deq.astype(np.float32))
    if fmt == rt.FMT_Q4:
        p, s = op.quant_q4(w, 32)
        tp, ts = dev(p), dev(s)
        deq = op.dequant_q4(p, s, 32)
        return rt.make_mat(fmt, N, K, tp, ts, group=32), [tp, ts], torch.from_numpy(deq.astype(np.float32))
    p, s, m = op.quant_q4a(w, 32)
    tp, ts, tm = dev(p), dev(s), dev(m)
    deq = op.dequant_q4a(p, s, m, 32)
    return rt.make_mat(fmt, N, K, tp, ts, tm, group=32), [tp, ts, tm], torch.from_numpy(deq.astype(np.float32))


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / max(b.norm().item(), 1e-30))


def anima_bind(h, W, norms, modA, modB, fmt=rt.FMT_F16, group=32, D=None, F=None, Cd=None):
    """Bind an Anima weight set (oracle naming) as device arrays; returns (wfd, operand weights, gain, keep)."""
    from oracle import anima as oa
    D = D or W["sq"].shape[0]
    F = F or W["m1"].shape[0]
    Cd = Cd or W["ck"].shape[1]
    fused = {rt.W_QKV: torch.cat((W["sq"], W["sk"], W["sv"]), 0), rt.W_O: W["so"], rt.W_CQ: W["cq"],
             rt.W_CKV: torch.cat((W["ck"], W["cv"]), 0), rt.W_CO: W["co"], rt.W_M1: W["m1"], rt.W_M2: W["m2"]}
    mats, keep, deq = {}, [], {}
    for slot, w in fused.items():
        m, k, d = make_mat(fmt, w.numpy(), group)
        mats[slot], deq[slot] = m, d
        keep += k
    Wd = {"sq": deq[rt.W_QKV][:D], "sk": deq[rt.W_QKV][D:2 * D], "sv": deq[rt.W_QKV][2 * D:], "so": deq[rt.W_O],
          "cq": deq[rt.W_CQ], "ck": deq[rt.W_CKV][:D], "cv": deq[rt.W_CKV][D:], "co": deq[rt.W_CO],
          "m1": deq[rt.W_M1], "m2": deq[rt.W_M2]}
    gain = oa.pack_gain(norms)
    tg, tA, tB = gain.cuda(), modA.cuda().contiguous(), modB.cuda().contiguous()
    keep += [tg, tA, tB]
    wfd = h.weights_bind(rt.MODEL_ANIMA, D, F, mats, tg, Cd=Cd, modA=tA, modB=tB, keep=keep)
    return wfd, Wd, gain, keep


def anima_blob(h, B, T, C, D, F, Cd):
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, Cd)
    bfd = h.buf_alloc(total)
    return meta, bfd


def write_f32(h, bfd, off, a):
    h.buf_write(bfd, off, np.ascontiguousarray(a, np.float32))


def read_f32(h, bfd, off, n):
    return np.frombuffer(h.buf_read(bfd, off, n * 4).tobytes(), np.float32).copy()


def dequant_q8_torch(u, s, group):
    """u8 [N][K] offset binary, fp16 scale [K/group][N] (CPU tensors) -> fp32 [N][K] = fp16(q * s): the same
    values as oracle.packs.dequant_q8 (q * s is exact in fp32, then one round to fp16), multithreaded."""
    N, K = u.shape
    q = u.view(N, K // group, group).to(torch.float32) - 128.0
    return (q * s.float().T.unsqueeze(-1)).half().float().view(N, K)


class LazyAnimaBlocks:
    """The oracle's view of synthetic device weight sets (hexanima_b200.synth): iterating yields
    (W, gain, modA, modB) per block in oracle naming, each rebuilt on the CPU from the device tensors when
    it is reached, so host memory holds one block's fp32 weights at a time (oracle.anima.sample iterates
    the blocks once per denoising step)."""

    def __init__(self, tensors, fmt, D, group=64):
        self.ts, self.fmt, self.D, self.group = tensors, fmt, D, group

    def __len__(self):
        return len(self.ts)

    def weights(self, i):
        t, D = self.ts[i], self.D
        deq = {}
        for slot, (w, s) in t["mats"].items():
            if self.fmt == rt.FMT_Q8:
                deq[slot] = dequant_q8_torch(w.cpu(), s.cpu(), self.group)
            else:
                deq[slot] = w.cpu().float()
        W = {"sq": deq[rt.W_QKV][:D], "sk": deq[rt.W_QKV][D:2 * D], "sv": deq[rt.W_QKV][2 * D:], "so": deq[rt.W_O],
             "cq": deq[rt.W_CQ], "ck": deq[rt.W_CKV][:D], "cv": deq[rt.W_CKV][D:], "co": deq[rt.W_CO],
             "m1": deq[rt.W_M1], "m2": deq[rt.W_M2]}
        return W, t["gain"].cpu().float(), t["modA"].cpu(), t["modB"].cpu()

    def __iter__(self):
        for i in range(len(self.ts)):
            yield self.weights(i)
