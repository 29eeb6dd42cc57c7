"""Generates tests/golden/rope_tables.json: RoPE inverse-frequency known answers.

The cases are the ones the reference pins (T/ = tests/HFLabs.ML.LLM.LevelZero.Tests/ of l0llm):
  - T/golden/rope.golden.json (default, linear4, yarn4_qwen3, yarn8_small, yarn2_explicit), checked by
    T/RopeFrequenciesTests.cs:25-47 with rel 1e-5;
  - the Llama-3.2-1B llama3 table inlined in T/RopeLlama3Tests.cs:8-38 (rel 1e-5);
  - plus the Llama-3-70B configuration this backend runs (llama3, factor 8, theta 5e5, head_dim 128).
Each table is recomputed here with Hugging Face transformers (ROPE_INIT_FUNCTIONS, the tool the
reference used) and, when the l0llm checkout is readable, compared with the reference's own golden
values before it is written. The fixture is what the tests read; the reference checkout is not needed
to run them.

Usage: python tests/golden/gen_rope_tables.py [--reference /path/to/l0llm]
"""
from __future__ import annotations

import argparse
import json
import re
from pathlib import Path

import torch
from transformers import LlamaConfig, Qwen3Config
from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

OUT = Path(__file__).resolve().parent / "rope_tables.json"

CASES = {
    "default": dict(head_dim=128, theta=1000000.0, max_pos=40960, scaling=None),
    "linear4": dict(head_dim=64, theta=10000.0, max_pos=2048, scaling={"rope_type": "linear", "factor": 4.0}),
    "yarn4_qwen3": dict(head_dim=128, theta=1000000.0, max_pos=131072,
                        scaling={"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}),
    "yarn8_small": dict(head_dim=64, theta=10000.0, max_pos=2048,
                        scaling={"rope_type": "yarn", "factor": 8.0, "original_max_position_embeddings": 2048}),
    "yarn2_explicit": dict(head_dim=64, theta=10000.0, max_pos=4096,
                           scaling={"rope_type": "yarn", "factor": 2.0, "original_max_position_embeddings": 2048,
                                    "beta_fast": 16.0, "beta_slow": 2.0, "attention_factor": 1.25}),
    "llama3_1b": dict(head_dim=64, theta=500000.0, max_pos=131072,
                      scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                               "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}),
    "llama3_70b": dict(head_dim=128, theta=500000.0, max_pos=131072,
                       scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}),
}


def compute(c: dict) -> tuple[list[float], float]:
    params = {"rope_theta": c["theta"]}
    params.update(c["scaling"] or {"rope_type": "default"})
    kind = params["rope_type"]
    if kind == "llama3":
        cfg = LlamaConfig(hidden_size=c["head_dim"] * 8, num_attention_heads=8, num_key_value_heads=4,
                          head_dim=c["head_dim"], max_position_embeddings=c["max_pos"], rope_parameters=params)
    else:
        cfg = Qwen3Config(hidden_size=c["head_dim"] * 8, num_attention_heads=8, num_key_value_heads=4,
                          head_dim=c["head_dim"], max_position_embeddings=c["max_pos"], rope_parameters=params)
    if kind == "default":
        inv, att = Qwen3RotaryEmbedding.compute_default_rope_parameters(cfg, "cpu")
    else:
        inv, att = ROPE_INIT_FUNCTIONS[kind](cfg, "cpu")
    return [float(x) for x in inv.tolist()], float(att)


def reference_tables(ref: Path) -> dict[str, list[float]]:
    """The reference's own values: rope.golden.json and the inline llama3 table (read as data)."""
    t = ref / "tests" / "HFLabs.ML.LLM.LevelZero.Tests"
    out = {}
    golden = t / "golden" / "rope.golden.json"
    if golden.exists():
        doc = json.loads(golden.read_text())
        for name, case in doc["cases"].items():
            out[name] = case["inv_freq"]
    cs = t / "RopeLlama3Tests.cs"
    if cs.exists():
        body = cs.read_text().split("Expected =", 1)[1].split("];", 1)[0]
        out["llama3_1b"] = [float(v) for v in re.findall(r"[-+]?\d\.\d+e[-+]\d+", body)]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the l0llm repository whose T/golden/rope.golden.json pins the tables")
    args = ap.parse_args()
    ref = reference_tables(Path(args.reference))
    doc = {"generator": "transformers " + __import__("transformers").__version__ + ", torch " + torch.__version__,
           "cases": {}}
    for name, c in CASES.items():
        inv, att = compute(c)
        if name in ref:
            want = ref[name]
            assert len(want) == len(inv), name
            worst = max(abs(a - b) / abs(b) for a, b in zip(inv, want))
            assert worst <= 1e-5, f"{name}: transformers and the reference golden differ by rel {worst}"
            print(f"{name}: matches the reference golden (max rel {worst:.2e})")
        doc["cases"][name] = {"head_dim": c["head_dim"], "theta": c["theta"], "max_position_embeddings": c["max_pos"],
                              "scaling": c["scaling"], "inv_freq": inv, "attention_factor": att,
                              "pinned_to_reference": name in ref}
    OUT.write_text(json.dumps(doc, indent=1))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
