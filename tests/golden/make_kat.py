"""Writes tests/golden/kat_cases.json: known-answer cases for the sampler.

Each expected id below is worked out by hand from the source text of
mini.js src/generation.js (pickToken :71-81, applyRepetitionPenalty :19-25,
argmax :51-55, softmaxTopNothing :9-17, sampleTopKTopP :27-49), not by running
any implementation.  The reasoning is stored with each case.  The logits are
chosen so every probability is exact (equal logits give exactly 1/n) or so the
answer depends on order alone.

    python tests/golden/make_kat.py
"""
import json
import os

NAN, INF, NINF = "nan", "inf", "-inf"


def P(do_sample=True, T=1.0, k=0, p=0.0, pen=1.0):
    return {"do_sample": do_sample, "temperature": T, "top_k": k, "top_p": p, "repetition_penalty": pen}


CASES = [
    # ---- greedy (argmax: first index of the strict max, NaN never wins)
    ("greedy_first_max", [1, 3, 3, 2], [], P(False), 0.0, 1,
     "argmax keeps the first 3 (index 1): 3 > 3 is false"),
    ("greedy_nan_at_0", [NAN, 5, 6], [], P(False), 0.0, 0,
     "logits[i] > NaN is false for every i, best stays 0"),
    ("greedy_nan_later", [1, NAN, 2], [], P(False), 0.0, 2, "NaN > 1 false; 2 > 1 true"),
    ("greedy_all_neg_inf", [NINF, NINF, NINF], [], P(False), 0.0, 0, "-inf > -inf is false"),
    ("greedy_low_temperature", [0, 7, 1], [], P(True, T=0.0001), 0.5, 1,
     "T <= 0.0001 takes the greedy branch even with do_sample"),
    # ---- penalty (Set semantics, OOB ids ignored, v>0 divides, v<=0 multiplies)
    ("penalty_divides_positive", [2.0, 0.5, -2.0], [0, 1, 1, 7, -3], P(False, pen=2.0), 0.0, 0,
     "work = [1.0, 0.25, -4.0]; duplicate 1 applied once; 7 and -3 out of range"),
    ("penalty_flips_greedy", [2.0, 1.5, -2.0], [0], P(False, pen=2.0), 0.0, 1,
     "work = [1.0, 1.5, -2.0]; argmax 1"),
    ("penalty_negative_multiplies", [-1.0, -1.5, -3.0], [0], P(False, pen=2.0), 0.0, 1,
     "work = [-2.0, -1.5, -3.0]; argmax 1"),
    ("penalty_one_is_off", [2.0, 1.5], [0], P(False, pen=1.0), 0.0, 0, "penalty 1.0 is skipped"),
    ("penalty_zero_is_off", [2.0, 1.5], [0], P(False, pen=0.0), 0.0, 0, "penalty 0 is falsy, skipped"),
    ("penalty_nan_is_off", [2.0, 1.5], [0], P(False, pen=NAN), 0.0, 0, "penalty NaN is falsy, skipped"),
    # ---- sampling over equal logits: probs exactly 0.25, identity order
    ("draw_u0", [0, 0, 0, 0], [], P(), 0.0, 0, "r = 0; 0 - 0.25 <= 0 at the first candidate"),
    ("draw_exact_boundary", [0, 0, 0, 0], [], P(), 0.25, 0, "r = 0.25; 0.25 - 0.25 = 0 <= 0"),
    ("draw_second", [0, 0, 0, 0], [], P(), 0.3, 1, "r = 0.3; 0.05 > 0; then -0.2 <= 0"),
    ("draw_last", [0, 0, 0, 0], [], P(), 0.999, 3, "r = 0.999 passes three boundaries"),
    ("topk_two", [0, 0, 0, 0], [], P(k=2), 0.6, 1, "cand [0,1], total 0.5, r = 0.3 -> index 1"),
    ("topk_ge_V_off", [0, 0, 0, 0], [], P(k=4), 0.999, 3, "topK < V is false: all 4 candidates"),
    ("topp_half", [0, 0, 0, 0], [], P(p=0.5), 0.9, 1,
     "acc 0.25, 0.5 >= 0.5 -> cut 2; total 0.5; r = 0.45 -> index 1"),
    ("topp_negative", [0, 0, 0, 0], [], P(p=-1.0), 0.999, 0, "acc 0.25 >= -1 -> cut 1"),
    ("topp_one_off", [0, 0, 0, 0], [], P(p=1.0), 0.999, 3, "topP < 1 false: no cut"),
    ("topp_zero_off", [0, 0, 0, 0], [], P(p=0.0), 0.999, 3, "topP 0 is falsy: no cut"),
    # ---- order: stable sort by prob desc keeps index order among ties
    ("tie_order_u0", [1, 2, 2, 1], [], P(), 0.0, 1, "sorted [1,2,0,3]: first is index 1"),
    ("tie_order_topk1", [1, 2, 2, 1], [], P(k=1), 0.999, 1, "top_k 1 keeps index 1 only"),
    ("tie_order_topk3_last", [1, 2, 2, 1], [], P(k=3), 0.999999, 0,
     "top_k 3 keeps [1,2,0]; u near 1 ends on index 0"),
    # ---- NaN probabilities: the fall-through returns the last candidate
    ("nan_logit_topk", [0, NAN, 0, 0], [], P(k=2), 0.5, 1,
     "sum is NaN; identity order; top_k 2 -> [0,1]; r NaN; last candidate 1"),
    ("nan_logit_full", [0, NAN, 0, 0], [], P(k=0, p=0.9), 0.5, 3,
     "no acc reaches topP; r NaN; last of all 4 candidates"),
    ("pos_inf_logit", [0, INF, 0], [], P(), 0.5, 2, "mx = inf gives inf - inf = NaN; last candidate"),
    ("all_neg_inf_sampled", [NINF, NINF], [], P(), 0.5, 1, "mx = -inf gives -inf - -inf = NaN"),
    ("temperature_nan", [0, 1, 2], [], P(T=NAN), 0.5, 2, "x / NaN = NaN everywhere"),
    # ---- single element
    ("single_element", [3.5], [], P(k=50, p=0.9), 0.7, 0, "V = 1"),
]


def main():
    out = []
    for name, logits, hist, params, u, expect, why in CASES:
        out.append({"name": name, "logits": logits, "hist": hist, "params": params, "u": u,
                    "expected_id": expect, "why": why})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat_cases.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(path, len(out))


if __name__ == "__main__":
    main()
