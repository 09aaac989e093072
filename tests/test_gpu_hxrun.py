"""hxrun: megarun's stdin protocol (hexagon/mega/megarun.cpp:132-195) on the GPU runtime, end to end
through files: two reference q8 block packs, one `run` line, output vs the oracle chain."""
import os
import subprocess

import numpy as np
import pytest
import torch

from hexanima_b200 import build
from oracle import anima as oa
from tests.gpu_util import rel

pytestmark = pytest.mark.gpu
D, CD, NCTX = 2048, 1024, 512


def _x32(rows, T):
    """[T][D] rows -> the reference's x32 tiles [T/32][D/32][32][32]."""
    return np.ascontiguousarray(rows.reshape(T // 32, 32, D // 32, 32).transpose(0, 2, 1, 3))


@pytest.mark.parametrize("x32", [False, True])
def test_hxrun_protocol_two_blocks(tmp_path, x32):
    exe = build._build_hxrun()
    sets = [oa.init_weights(200 + i, D=D, F=8192, Cd=CD) for i in range(2)]
    packs = []
    for i, (W, norms, modA, modB) in enumerate(sets):
        pack = oa.build_pack(W, norms, modA, modB, q8=True)
        (tmp_path / f"blk{i:02d}.bin").write_bytes(pack)
        packs.append(pack)
    gh, gw = 16, 32
    T = gh * gw
    g = torch.Generator().manual_seed(9)
    x = torch.randn(T, D, generator=g)
    emb = torch.randn(D, generator=g)
    lora = torch.randn(3 * D, generator=g) * 0.1
    ctx = torch.randn(NCTX, CD, generator=g)
    xin = tmp_path / ("x_in.x32" if x32 else "x_in.raw")
    xout = tmp_path / ("x_out.x32" if x32 else "x_out.raw")
    (_x32(x.numpy(), T) if x32 else x.numpy().T.copy()).astype(np.float32).tofile(xin)
    emb.numpy().astype(np.float32).tofile(tmp_path / "emb.raw")
    lora.numpy().astype(np.float32).tofile(tmp_path / "lora.raw")
    ctx.numpy().T.astype(np.float32).copy().tofile(tmp_path / "ctx.raw")   # [1024 ch][512 tok]
    p = subprocess.Popen([exe, str(tmp_path), "0", "2"], stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                         stderr=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == "ready"
        p.stdin.write(f"run {xin} {tmp_path}/emb.raw {tmp_path}/lora.raw {tmp_path}/ctx.raw {xout} {gh} {gw}\n")
        p.stdin.flush()
        line = p.stdout.readline().strip()
        assert line.startswith("done"), (line, p.stderr.read() if p.poll() is not None else "")
        p.stdin.write(f"run {tmp_path}/missing.raw {tmp_path}/emb.raw {tmp_path}/lora.raw {tmp_path}/ctx.raw "
                      f"{xout}.2\n")
        p.stdin.flush()
        assert p.stdout.readline().strip() == "error"
        p.stdin.write("quit\n")
        p.stdin.flush()
        assert p.wait(timeout=120) == 0
    finally:
        if p.poll() is None:
            p.kill()
    out = np.fromfile(xout, np.float32)
    got = out.reshape(T // 32, D // 32, 32, 32).transpose(0, 2, 1, 3).reshape(T, D) if x32 else out.reshape(D, T).T
    c, s = oa.make_rope(gh, gw)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    xr = x[None].clone()
    ctx16 = ctx.half().float()[None]
    for (W, norms, modA, modB), pack in zip(sets, packs):
        Wd, gain = oa.pack_weights(pack, q8=True)
        xr = oa.block(xr, ctx16, oa.modulation(modA, modB, emb, lora), cos, sin, Wd, gain)
    assert rel(torch.from_numpy(np.ascontiguousarray(got))[None] - x[None], xr - x[None]) < 2e-3
