"""Generate the golden vectors that pin the oracle to the reference implementation.

Run in a container that has the reference checkout (its path in HX_REFERENCE, else the default
below); the committed .npz files are what the tests read, so the reference is not needed to run the
tests.

  python tests/golden/make_golden.py

What is run from the reference (its code, not a restatement):
  moss/export_all_q8.py         wt16, q8tiles (MOSS scale floor)
  hexagon/mega/export_all.py    wt16, q8tiles (Anima scale floor); the module runs main() on import,
                                so the two functions are compiled out of its source with ast
  moss/mkblk_test.py            unpack (q8 record decode); module-level code loads model files, so
                                the function is compiled out of its source with ast
  moss/export_te.py             q4a_tiles, unpack_q4a
  moss/moss_ref.py              block, rope_tables on seeded synthetic weights (lora off and on);
                                text_block, text_refine and time_vecs (moss_text.npz)
"""
import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("HX_REFERENCE", "/root/reference")
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def functions_from(path, names, extra_globals):
    """Compile only the named top-level function definitions of a source file."""
    tree = ast.parse(open(path).read(), path)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    mod = ast.Module(body=keep, type_ignores=[])
    ns = dict(extra_globals)
    exec(compile(mod, path, "exec"), ns)
    return {n: ns[n] for n in names}


def main():
    sys.path.insert(0, os.path.join(REF, "moss"))
    import export_all_q8 as q8m  # noqa: E402
    import export_te  # noqa: E402
    import moss_ref  # noqa: E402

    anima = functions_from(os.path.join(REF, "hexagon/mega/export_all.py"), ["wt16", "q8tiles"], {"np": np})
    mk = functions_from(os.path.join(REF, "moss/mkblk_test.py"), ["unpack"], {"np": np, "torch": torch})

    # ------------------------------------------------------------ pack codecs
    rng = np.random.default_rng(20261201)
    K, N = 96, 128
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    W[:, 5] = 0.0                 # all-zero column: Anima floor 1.0, MOSS floor 6.2e-5
    W[:32, 9] = 1e-7              # tiny column in the first k tile: denormal scale before the floor
    W[40, 17] = 0.9               # one outlier
    t_moss = q8m.wt16(W)
    t_anima = anima["wt16"](W)
    q8_moss = q8m.q8tiles(t_moss)
    q8_anima = anima["q8tiles"](t_anima)
    unpack_moss = mk["unpack"](q8_moss, N // 32, K // 32).numpy()
    qn = rng.integers(0, 16, size=(N, K)).astype(np.uint8)       # [out][in] nibbles
    S = (np.abs(rng.standard_normal((N, K // 32))) * 0.01 + 1e-3).astype(np.float32)
    M = (rng.standard_normal((N, K // 32)) * 0.05).astype(np.float32)
    q4a = export_te.q4a_tiles(qn, S, M)
    unpack_q4a = export_te.unpack_q4a(q4a, N // 32, K // 32)
    np.savez_compressed(os.path.join(HERE, "packs.npz"), W=W, wt16=np.frombuffer(t_moss.tobytes(), np.uint8),
                        q8_moss=np.frombuffer(q8_moss, np.uint8), q8_anima=np.frombuffer(q8_anima, np.uint8),
                        unpack_moss=unpack_moss, q4_nib=qn, q4_S=S, q4_M=M, q4a=np.frombuffer(q4a, np.uint8),
                        unpack_q4a=unpack_q4a)

    # ------------------------------------------------------------ MOSS block (moss_ref.block)
    from oracle import moss as om  # the generator of the synthetic inputs, shared with the tests

    torch.set_grad_enabled(False)
    D, F, Hh, Ww, T = 3072, 256, 2, 4, 16
    Nt = Hh * Ww + T
    bands = om.bands16()
    sin, cos = moss_ref.rope_tables(Hh, Ww, T, bands)
    out = {"D": D, "F": F, "H": Hh, "W": Ww, "T": T, "bands": bands.numpy(), "sin": sin.numpy(), "cos": cos.numpy()}
    for tag, rank, seed in (("plain", 0, 11), ("lora", 8, 12)):
        w, lora = om.init_weights(seed, D=D, F=F, lora_rank=rank)
        gen = torch.Generator().manual_seed(seed + 100)
        x = torch.randn(Nt, D, generator=gen)
        mod = torch.randn(6, D, generator=gen) * 0.1
        y = moss_ref.block(x, mod, sin, cos, lambda n: w[n], 0, (lambda i, n: lora[n]) if rank else None)
        out[f"{tag}_seed"] = seed
        out[f"{tag}_x_sum"] = float(x.double().sum())
        out[f"{tag}_w_sum"] = float(sum(v.double().sum() for v in w.values()))
        out[f"{tag}_out"] = y.numpy()
    np.savez_compressed(os.path.join(HERE, "moss_block.npz"), **out)

    # ------------------------------------------------------------ MOSS text side (moss_ref.text_block / text_refine /
    # time_vecs): refiner at D 3072 (24 heads are fixed in moss_ref.attn), FFN 256; time_vecs at D 256
    Tt = 20
    s_t, c_t = moss_ref.rope_tables(0, 1, Tt, bands)           # text rows only: coords (0, i, 0, 0)
    wt = om.init_text_weights(21, D=3072, F=256)
    gen = torch.Generator().manual_seed(121)
    xt = torch.randn(Tt, 3072, generator=gen)
    txt = torch.randn(Tt, 4096, generator=gen)
    g = lambda n: wt[n]
    tb = moss_ref.text_block(xt, "text_embedder.blocks.0.", s_t, c_t, g)
    tr = moss_ref.text_refine(txt, s_t, c_t, g)
    wtime = om.init_time_weights(22, D=256)
    mod, head = moss_ref.time_vecs(968.0, lambda n: wtime[n])
    np.savez_compressed(os.path.join(HERE, "moss_text.npz"), T=Tt, text_seed=21, time_seed=22, t_code=968.0,
                        x=xt.numpy(), txt=txt.numpy(), sin=s_t.numpy(), cos=c_t.numpy(), text_block=tb.numpy(),
                        text_refine=tr.numpy(), mod=mod.numpy(), head=head.numpy())
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
