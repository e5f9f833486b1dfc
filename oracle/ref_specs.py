"""Bench/parity sample shapes for which oracle/build_ref.py compiles the
reference's own CPU library (TEST INFRASTRUCTURE ONLY).

Each spec is one unit of a BASELINE config: the slice of the workload that one
call of a shape-specialised reference library computes (the reference CPU
path is JIT-compiled per shape, builder.py:606-736). `units` says how many such
slices make up the full config, so a rate measured on slices scales to the
config's own metric.
"""

SPECS = {
    # name: (equation, shape0, shape1, units per full config, config)
    "cfg1": ("ij,jk->ik", (256, 256), (256, 256), 1, "cfg1"),
    "cfg2_b1": ("bij,bjk->bik", (1, 1024, 1024), (1, 1024, 1024), 64, "cfg2"),
    "cfg3_bh1": ("bshd,bthd->bsht", (1, 2048, 1, 128), (1, 2048, 1, 128), 256, "cfg3"),
    "cfg3u_bh1": ("bshd,bthd->bsht", (1, 2000, 1, 80), (1, 2000, 1, 80), 256, "cfg3u"),
    "cfg4a_t512": ("tn,sn->ts", (512, 128), (8192, 128), 16, "cfg4a"),
    "cfg4b_t512": ("ts,ts->ts", (512, 8192), (512, 8192), 16, "cfg4b"),
    "cfg4c_t512": ("ts,sp->tp", (512, 8192), (8192, 128), 16, "cfg4c"),
    "cfg5_rms_b1": ("bsd,d->bsd", (1, 4096, 4096), (4096,), 16, "cfg5_rms"),
    "cfg5_rope_b1": ("bshd,sd->bshd", (1, 4096, 32, 128), (4096, 128), 16, "cfg5_rope"),
    "cfg5_alibi_h1": ("hqk,h->hqk", (1, 4096, 4096), (1,), 32, "cfg5_alibi"),
}
