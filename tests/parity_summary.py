"""Summarises the parity log the GPU block tests write ($ASTRO_PARITY_LOG, one JSON
line per compared block call) as the markdown table kept in profiles/.

    ASTRO_PARITY_LOG=parity.jsonl python -m pytest tests/test_gpu_block.py -m gpu
    python tests/parity_summary.py parity.jsonl
"""
from __future__ import annotations

import json
import sys


def summarise(lines) -> str:
    rows = [json.loads(l) for l in lines if l.strip()]
    groups = {}
    for r in rows:
        k = (r["case"], r["kernels"]["router"], r["kernels"]["experts"], r["kernels"]["shared_expert"])
        g = groups.setdefault(k, dict(calls=0, rows=0, differ=0, outputs=0, logits_c=0, sets_c=0,
                                      beyond_c=0, differ_c=0, raw_c=0.0, scaled_c=0.0, rel_c=0.0,
                                      T=set()))
        g["calls"] += 1
        g["rows"] += r["rows"]
        g["T"].add(r["T"])
        g["differ"] += r["exact"]["n_differ"]
        g["outputs"] += r["exact"]["n"]
        c = r.get("canonical")
        if c:
            g["logits_c"] += r["canonical_logits_differ"]
            g["sets_c"] += r["canonical_expert_sets_differ"]
            g["beyond_c"] += c["n_beyond"]
            g["differ_c"] += c["n_differ"]
            g["raw_c"] = max(g["raw_c"], c["raw_max_abs"])
            g["scaled_c"] = max(g["scaled_c"], c["scaled_max_abs"])
            g["rel_c"] = max(g["rel_c"], c["rel_l2"])
    out = ["| case | T | router kernel | expert kernel | shared-expert kernel | calls | rows | "
           "outputs differing from the oracle (same arithmetic) | canonical order: logits "
           "differing | expert sets differing | outputs differing | beyond 2e-2·max(\\|e\\|,1) | "
           "raw max-abs | scaled max-abs | rel-L2 |",
           "|---|---|---|---|---|---:|---:|---:|---:|---:|---:|---:|---:|---:|---:|"]
    for (case, router, experts, shared), g in groups.items():
        ts = ",".join(str(t) for t in sorted(g["T"]))
        out.append(f"| {case} | {ts} | {router} | {experts} | {shared} | {g['calls']} | {g['rows']} | "
                   f"{g['differ']} of {g['outputs']} | {g['logits_c']} | {g['sets_c']} | "
                   f"{g['differ_c']} | {g['beyond_c']} | {g['raw_c']:.4g} | {g['scaled_c']:.4g} | "
                   f"{g['rel_c']:.3g} |")
    return "\n".join(out) + "\n"


if __name__ == "__main__":
    with open(sys.argv[1]) as f:
        sys.stdout.write(summarise(f))
