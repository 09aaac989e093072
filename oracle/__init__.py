"""CPU oracle for the DiT block path — TEST INFRASTRUCTURE ONLY.

A plain numpy / torch-fp32 restatement of the reference's algorithms, each function citing the
reference file:line it follows. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
and reference legs may import it, and only as the checker or the timed CPU baseline; the product
(hexanima_b200, libhxdit.so) never calls it.

Pinning:
  * packs.py  (q8 / q4a tile records, unpack) is pinned bit-exactly against golden vectors that
    tests/golden/make_golden.py produced by running the reference's own export_all_q8.py,
    hexagon/mega/export_all.py, mkblk_test.py and export_te.py code.
  * moss.py  (MOSS block, RoPE tables) is pinned against moss/moss_ref.py outputs (same script).
  * anima.py (Anima block): the reference ships no runnable Anima block (export_block.py imports
    the absent phase0_block / block_test); the restatement of hexagon/mega/blk.c:148-175 is the
    contract — parity unpinned at block level. Its pieces shared with moss.py (RMS, RoPE rotation,
    attention) are pinned through the MOSS vectors.
"""
