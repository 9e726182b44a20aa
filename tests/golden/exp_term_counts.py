"""How often the choice of Math.exp changes the reference's softmax terms.

For every row of the five sampling workloads (the same seeded generators the
tests and the benchmark use), the oracle builds the row exactly as
src/generation.js:72-79 does (penalty, temperature), then computes each term
fp32(exp(x - mx)) of src/generation.js:14 twice: with V8's Math.exp (the fdlibm
method, the oracle's default) and with the C library's exp.  Writes the counts
to exp_term_counts.json next to this file.

    python tests/golden/exp_term_counts.py [--rows N]

Test infrastructure: it measures the oracle, it is not part of the product.
"""
import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "omni.js_b200"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=0, help="rows per workload (0: the whole batch)")
    args = ap.parse_args()
    import ms_oracle
    from minisample import workloads as W

    ms_oracle.build()
    ms_oracle.set_exp(libc=False)
    out = {}
    for name in ("gpt2_b1", "llama3_b64", "qwen2_b256", "gemma_b512", "vocab_sharded"):
        w = W.WORKLOADS[name]
        B = w.B if args.rows <= 0 else min(args.rows, w.B)
        if name == "gpt2_b1":  # one row per step: 256 steps of fresh logits
            X = np.concatenate([W.logits_np(w, 1000 + s, B=1) for s in range(w.steps)])
            hist, off = None, None
        else:
            X = W.logits_np(w, 5, B=B)
            hist, off = W.history_np(w, 5, B=B)
        p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                                  w.params.repetition_penalty)
        terms = diff = rows_hit = 0
        for r in range(X.shape[0]):
            h = None if hist is None else hist[off[r]:off[r + 1]]
            _, d, work, _ = ms_oracle.pick_token(X[r], h, p, 0.5, want_arrays=True)
            a, b = ms_oracle.terms_both(work, float(d["mx"]))
            n = int(np.sum(a.view(np.uint32) != b.view(np.uint32)))
            terms += work.shape[0]
            diff += n
            rows_hit += n > 0
        out[name] = {"rows": int(X.shape[0]), "terms": int(terms), "terms_differing": int(diff),
                     "rows_with_a_difference": int(rows_hit)}
        print(name, out[name], flush=True)
    with open(os.path.join(HERE, "exp_term_counts.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
