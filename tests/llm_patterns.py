"""Two-operand contraction patterns of LLM layers, as listed by the reference's
benchmarks/complex/bench_llm_contractions.py:214-258 (equations only; the
sizes here are this project's own). Used by the GPU parity tests (tiny sizes)
and by bench.py --suite callers (LLM-scale sizes)."""

# name, equation, operand 0 axes sizes, operand 1 axes sizes (by label)
PATTERNS = [
    ("batched_linear", "bsi,oi->bso"),
    ("attention_scores", "bshd,bthd->bsht"),
    ("attention_context", "bsht,bthd->bshd"),
    ("output_projection", "bshd,hdo->bso"),
    ("rope", "bshd,sd->bshd"),
    ("swiglu_up", "bsi,fi->bsf"),
    ("swiglu_down", "bsf,if->bsi"),
    ("lora_a", "bsi,ir->bsr"),
    ("lora_b", "bsr,ro->bso"),
    ("pairwise_similarity", "bd,cd->bc"),
    ("moe_router", "bsi,ei->bse"),
    ("moe_expert", "bsi,eio->bseo"),
    ("moe_combine", "bse,bseo->bso"),
    ("rotary_matrix", "bshd,hdk->bshk"),
    ("linear_dense", "bsd,de->bse"),
    ("batched_outer", "bi,bj->bij"),
    ("headwise_qkv", "bsd,hde->bshe"),
    ("lora_update", "bsr,rd->bsd"),
    ("moe_dispatch", "bse,bek->bsk"),
    ("rms_norm", "bsd,d->bsd"),
    ("quadform_1", "bi,ij->bj"),
    ("quadform_2", "bj,j->b"),
    ("token_pos_embed", "bsd,sd->bsd"),
    ("alibi_bias", "hqk,h->hqk"),
    ("logits", "bsd,vd->bsv"),
]

SMALL = dict(b=2, s=24, t=24, h=4, d=32, i=48, o=40, f=56, r=8, c=36, e=4, k=16, v=72, j=20, q=24)
LARGE = dict(b=4, s=2048, t=2048, h=32, d=128, i=4096, o=4096, f=11008, r=16, c=8192, e=8, k=128,
             v=32000, j=4096, q=2048)


def shapes(eq, sizes):
    lhs = eq.split("->")[0].split(",")
    return tuple(tuple(sizes[ch] for ch in op) for op in lhs)
