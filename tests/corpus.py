"""Parity corpus: equations and shapes exercised by the reference test suite and
by BASELINE.json's configs.

Sources (case lists, not code):
  * EINSUM_CASES     tests/test_einsum.py:22-128 (every kernel routing branch)
  * ATTENTION_CASES  tests/test_llm_ops.py:34-62
  * BROADCAST_CASES  tests/test_llm_ops.py:115-125
  * CHAIN_CASES      tests/test_llm_ops.py:81-107 (linear-attention chain steps)
  * BATCHED_PARTIAL  tests/test_einsum.py:161-167 (rejected by the reference planner)
  * CONFIGS          BASELINE.json configs 1-5 (full sizes)
"""

EINSUM_CASES = [
    # identity-layout matmul
    ("ij, jk -> ik", (32, 64), (64, 128)),
    ("ij, jk -> ik", (256, 256), (256, 384)),
    ("i, j -> ij", (64,), (96,)),
    ("i, i -> ", (256,), (256,)),
    ("ij, j -> i", (32, 64), (64,)),
    ("i, ij -> j", (32,), (32, 64)),
    ("ij, jk -> ik", (16, 2048), (2048, 16)),
    ("ijk, jkl -> il", (8, 16, 32), (16, 32, 64)),
    # transposed inputs
    ("ji, jk -> ik", (64, 32), (64, 128)),
    ("ij, kj -> ik", (32, 64), (128, 64)),
    ("ji, kj -> ik", (64, 32), (128, 64)),
    ("ji, jk -> ik", (512, 500), (512, 64)),
    # non-identity output permutation
    ("ij, jk -> ki", (32, 64), (64, 48)),
    ("ai, ja -> ij", (32, 16), (64, 32)),
    ("abc, cd -> abd", (32, 16, 32), (32, 64)),
    # fused output permutation
    ("bshd, bthd -> bsht", (2, 128, 4, 64), (2, 128, 4, 64)),
    ("bshd, bthd -> bsht", (2, 64, 4, 32), (2, 96, 4, 32)),
    ("bsht, bthd -> bshd", (2, 128, 4, 128), (2, 128, 4, 64)),
    ("shd, thd -> sht", (200, 1, 64), (128, 1, 64)),
    # batched
    ("bij, bjk -> bik", (32, 16, 32), (32, 32, 64)),
    ("bji, bjk -> bik", (24, 32, 16), (24, 32, 64)),
    ("bij, bjk -> bik", (64, 128, 128), (64, 128, 128)),
    ("bshd, bthd -> bsht", (2, 128, 16, 64), (2, 128, 16, 64)),
    # NT direct read
    ("bihd, bjhd -> bihj", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("bihd, bjhd -> bihj", (4, 128, 4, 128), (4, 128, 4, 128)),
    ("bnd, bmd -> bnm", (8, 128, 64), (8, 128, 64)),
    ("bihd, bjhd -> bihj", (2, 64, 4, 32), (2, 96, 4, 32)),
    # NN-strided direct read
    ("bihj, bjhd -> bihd", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("bihj, bjhd -> bihd", (4, 128, 4, 128), (4, 128, 4, 128)),
    ("bvhd, bhde -> bvhe", (4, 128, 8, 64), (4, 8, 64, 64)),
    ("bnj, bjm -> bnm", (8, 128, 128), (8, 128, 64)),
    # TN direct read
    ("bvhd, bvhe -> bhde", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("bvhd, bvhe -> bhde", (4, 128, 4, 64), (4, 128, 4, 64)),
    ("vnd, vne -> nde", (128, 8, 64), (128, 8, 64)),
    # K != C
    ("ij, jk -> ik", (32, 20), (20, 128)),
    ("ai, ja -> ij", (20, 16), (64, 20)),
    ("ji, jk -> ik", (20, 32), (20, 128)),
    ("bij, bjk -> bik", (8, 16, 20), (8, 20, 64)),
    # elementwise
    ("i, i -> i", (1000,), (1000,)),
    ("ts, ts -> ts", (64, 48), (64, 48)),
    ("bshd, bshd -> bshd", (2, 16, 8, 64), (2, 16, 8, 64)),
    # partial output tiles
    ("ij, jk -> ik", (250, 128), (128, 256)),
    ("ij, jk -> ik", (256, 128), (128, 250)),
    ("ij, jk -> ik", (250, 128), (128, 250)),
    # partial tile grid
    ("ij, jk -> ik", (200, 64), (64, 128)),
    ("ij, jk -> ik", (128, 64), (64, 200)),
    ("ij, jk -> ik", (200, 64), (64, 200)),
    ("ij, jk -> ik", (1000, 64), (64, 128)),
    ("ij, jk -> ik", (200, 20), (20, 200)),
]

ATTENTION_CASES = [
    ("bshd, bthd -> bsht", (4, 16, 8, 64), (4, 16, 8, 64)),
    ("bsht, bthd -> bshd", (4, 16, 8, 16), (4, 16, 8, 64)),
    ("bshd, hdk -> bshk", (4, 16, 8, 64), (8, 64, 64)),
    ("bhs, bht -> bst", (1, 20, 16), (1, 20, 24)),
    ("bhs, bht -> bst", (4, 20, 16), (4, 20, 24)),
    ("bhsc, bcht -> bsht", (2, 8, 16, 20), (2, 20, 8, 24)),
    ("bhsc, bhtc -> bhst", (2, 8, 16, 20), (2, 8, 24, 20)),
    ("bhs, bht -> bst", (2, 128, 256), (2, 128, 64)),
    ("bhs, bht -> bst", (2, 130, 256), (2, 130, 64)),
    ("bhsc, bhtc -> bhst", (2, 4, 16, 130), (2, 4, 256, 130)),
]

BROADCAST_CASES = [
    ("bsd, d -> bsd", (2, 8, 64), (64,)),
    ("bsd, sd -> bsd", (2, 8, 64), (8, 64)),
    ("bshd, sd -> bshd", (2, 8, 4, 16), (8, 16)),
    ("hqk, h -> hqk", (8, 16, 16), (8,)),
    ("bsd, d -> bsd", (2, 16, 512), (512,)),
    ("bshd, sd -> bshd", (4, 32, 8, 64), (32, 64)),
]

CHAIN_CASES = []
for _T, _N, _P in ((96, 64, 128), (320, 64, 128)):
    CHAIN_CASES += [("tn, sn -> ts", (_T, _N), (_T, _N)),
                    ("ts, ts -> ts", (_T, _T), (_T, _T)),
                    ("ts, sp -> tp", (_T, _T), (_T, _P))]

BATCHED_PARTIAL = [("bij, bjk -> bik", (4, 200, 64), (4, 64, 128))]

# BASELINE.json configs (name, equation, shape0, shape1, dtype name)
CONFIGS = [
    ("cfg1", "ij,jk->ik", (256, 256), (256, 256), "float32"),
    ("cfg2", "bij,bjk->bik", (64, 1024, 1024), (64, 1024, 1024), "float16"),
    ("cfg3", "bshd,bthd->bsht", (8, 2048, 32, 128), (8, 2048, 32, 128), "float16"),
    ("cfg3u", "bshd,bthd->bsht", (8, 2000, 32, 80), (8, 2000, 32, 80), "float16"),
    ("cfg4a", "tn,sn->ts", (8192, 128), (8192, 128), "float32"),
    ("cfg4b", "ts,ts->ts", (8192, 8192), (8192, 8192), "float32"),
    ("cfg4c", "ts,sp->tp", (8192, 8192), (8192, 128), "float32"),
    ("cfg5_rms", "bsd,d->bsd", (16, 4096, 4096), (4096,), "float16"),
    ("cfg5_rope", "bshd,sd->bshd", (16, 4096, 32, 128), (4096, 128), "float16"),
    ("cfg5_alibi", "hqk,h->hqk", (32, 4096, 4096), (32,), "float16"),
]

ALL_SMALL = EINSUM_CASES + ATTENTION_CASES + BROADCAST_CASES + CHAIN_CASES + BATCHED_PARTIAL


def case_id(eq, s0, s1):
    e = eq.replace(" ", "").replace(",", "_").replace("->", "-")
    return f"{e}[{'x'.join(map(str, s0))}|{'x'.join(map(str, s1))}]"
