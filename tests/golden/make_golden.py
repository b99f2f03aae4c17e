"""Extracts the reference's own golden vectors into compact test fixtures.

Run once on a machine that has the Kestrel-Q tree (its location is the
--reference argument); the outputs are committed so that tests never read
the reference at run time:

  gdn_golden.npz / gdn_golden.json   research/operators/.../gdn-{contract,
                                     calibration,holdout,state-vectors,
                                     native-validation}.json
  qsa_golden.npz / qsa_golden.json   research/operators/.../qsa-{contract,
                                     calibration,holdout,state-vectors,
                                     selection-vectors,native-validation}.json
  moe_golden.npz / moe_golden.json   research/operators/.../moe-{contract,
                                     calibration,holdout,routing-vectors,
                                     native-validation}.json
  layer_golden.npz / layer_golden.json
                                     research/operators/.../layer-{contract,
                                     calibration,holdout,native-validation}.json
  dequant_golden.json                research/numerics/.../dequant-vectors.json

Expected values in those files come from pinned Transformers / llama.cpp
oracles (never from Kestrel-Q itself); the calibrated abs / rel / ULP
contracts are copied alongside.  Usage:
  python tests/golden/make_golden.py [--reference <Kestrel-Q checkout>]
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

REV = "de4b8e4d43b917e7706784d8bb445c9af86a3540"
OUT = Path(__file__).resolve().parent


def f32(record) -> np.ndarray:
    raw = b"".join(bytes.fromhex(h) for h in record["f32_le_hex"])
    return np.frombuffer(raw, dtype="<f4").reshape(record["shape"]).astype(np.float32)


def gdn(ops: Path) -> None:
    contract = json.loads((ops / "gdn-contract.json").read_text())
    cal = json.loads((ops / "gdn-calibration.json").read_text())
    hold = json.loads((ops / "gdn-holdout.json").read_text())
    chain = json.loads((ops / "gdn-state-vectors.json").read_text())
    native = json.loads((ops / "gdn-native-validation.json").read_text())
    arrays: dict[str, np.ndarray] = {}
    w = contract["weights"]
    names = {"a_log": "A_log", "conv": "conv1d.weight", "dt_bias": "dt_bias", "alpha": "in_proj_a.weight",
             "beta": "in_proj_b.weight", "qkv": "in_proj_qkv.weight", "gate": "in_proj_z.weight",
             "norm": "norm.weight", "output": "out_proj.weight"}
    for k, v in names.items():
        arrays[f"w_{k}"] = f32(w[v]).reshape(-1)
    cases = []
    for split, src in (("calibration", cal["cases"]), ("holdout", hold["cases"])):
        for c in src:
            i = len(cases)
            arrays[f"c{i}_input"] = f32(c["input"]).reshape(-1, contract["reduced_config"]["hidden_size"])
            arrays[f"c{i}_conv0"] = f32(c["initial_state"]["conv"]).reshape(-1)
            arrays[f"c{i}_rec0"] = f32(c["initial_state"]["recurrent"]).reshape(-1)
            arrays[f"c{i}_output"] = f32(c["expected"]["output"]).reshape(-1)
            arrays[f"c{i}_conv"] = f32(c["expected"]["conv_state"]).reshape(-1)
            arrays[f"c{i}_rec"] = f32(c["expected"]["recurrent_state"]).reshape(-1)
            cases.append({"id": c["id"], "split": split, "mask": c.get("padding_mask"),
                          "initialized": bool(c["initial_state"]["initialized"])})
    # prefix -> decode -> decode chain, and its full recomputation
    pre = chain["prefill"]
    arrays["chain_prefix_input"] = f32(pre["input"]).reshape(-1, contract["reduced_config"]["hidden_size"])
    arrays["chain_prefix_output"] = f32(pre["expected"]["output"]).reshape(-1)
    for j, step in enumerate(chain["decode_steps"]):
        arrays[f"chain_step{j}_input"] = f32(step["input"]).reshape(-1, contract["reduced_config"]["hidden_size"])
        arrays[f"chain_step{j}_output"] = f32(step["expected_output"]).reshape(-1)
        arrays[f"chain_step{j}_conv"] = f32(step["expected_conv_state"]).reshape(-1)
        arrays[f"chain_step{j}_rec"] = f32(step["expected_recurrent_state"]).reshape(-1)
    full = chain["full_recomputation"]
    arrays["chain_full_input"] = f32(full["input"]).reshape(-1, contract["reduced_config"]["hidden_size"])
    arrays["chain_full_output"] = f32(full["expected"]["output"]).reshape(-1)
    contracts = {k: {kk: v[kk] for kk in ("comparison_class", "abs_limit", "rel_limit", "ulp_limit")}
                 for k, v in native["contracts"].items()}
    meta = {"source": f"Kestrel-Q research/operators/Qwen3.8-Flash-Next/{REV}/gdn-*.json",
            "expected_values_source": cal["expected_values_source"], "oracle": cal["oracle"],
            "reduced_config": contract["reduced_config"], "cases": cases,
            "chain_steps": len(chain["decode_steps"]), "contracts": contracts}
    np.savez_compressed(OUT / "gdn_golden.npz", **arrays)
    (OUT / "gdn_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


def qsa(ops: Path) -> None:
    contract = json.loads((ops / "qsa-contract.json").read_text())
    cal = json.loads((ops / "qsa-calibration.json").read_text())
    hold = json.loads((ops / "qsa-holdout.json").read_text())
    chain = json.loads((ops / "qsa-state-vectors.json").read_text())["cases"][0]
    selv = json.loads((ops / "qsa-selection-vectors.json").read_text())
    native = json.loads((ops / "qsa-native-validation.json").read_text())
    rc = contract["reduced_config"]
    H = rc["hidden_size"]
    w = contract["weights"]
    arrays: dict[str, np.ndarray] = {}
    qk = f32(w["indexer.index_qk_proj.weight"]).reshape(-1)
    iq_count = rc["index_query_heads"] * rc["index_head_dim"] * H
    arrays["w_query"] = f32(w["q_proj.weight"]).reshape(-1)
    arrays["w_key"] = f32(w["k_proj.weight"]).reshape(-1)
    arrays["w_value"] = f32(w["v_proj.weight"]).reshape(-1)
    arrays["w_output"] = f32(w["o_proj.weight"]).reshape(-1)
    arrays["w_query_norm"] = f32(w["q_norm.weight"]).reshape(-1)
    arrays["w_key_norm"] = f32(w["k_norm.weight"]).reshape(-1)
    arrays["w_index_query"] = qk[:iq_count]
    arrays["w_index_key"] = qk[iq_count:]
    arrays["w_index_query_norm"] = f32(w["indexer.q_layernorm.weight"]).reshape(-1)
    arrays["w_index_key_norm"] = f32(w["indexer.k_layernorm.weight"]).reshape(-1)

    def state_arrays(prefix, st):
        arrays[f"{prefix}_key"] = f32(st["key"]).reshape(st["length"], -1) if st["length"] else np.zeros((0, 1), np.float32)
        arrays[f"{prefix}_value"] = f32(st["value"]).reshape(st["length"], -1) if st["length"] else np.zeros((0, 1), np.float32)
        arrays[f"{prefix}_raw"] = f32(st["raw_index_key"]).reshape(st["length"], -1) if st["length"] else np.zeros((0, 1), np.float32)

    def selection_list(prefix, sels):
        out = []
        for j, s in enumerate(sels):
            arrays[f"{prefix}_sel{j}_scores"] = f32(s["candidate_scores"]).reshape(-1) if s["candidate_scores"]["f32_le_hex"] else np.zeros(0, np.float32)
            out.append({"absolute_position": s["absolute_position"], "selected_block_ids": s["selected_block_ids"],
                        "selected_token_positions": s["selected_token_positions"],
                        "tail_positions": s["tail_positions"]})
        return out

    cases = []
    for split, src in (("calibration", cal["cases"]), ("holdout", hold["cases"])):
        for c in src:
            i = len(cases)
            arrays[f"c{i}_input"] = f32(c["input"]).reshape(-1, H)
            arrays[f"c{i}_output"] = f32(c["expected"]["output"]).reshape(-1)
            state_arrays(f"c{i}_state", c["expected"]["state"])
            cases.append({"id": c["id"], "split": split, "length": c["expected"]["state"]["length"],
                          "selection": selection_list(f"c{i}", c["expected"]["selection"])})
    arrays["chain_prefix_input"] = f32(chain["prefix_input"]).reshape(-1, H)
    state_arrays("chain_prefix_state", chain["prefix_state"])
    steps = []
    for j, step in enumerate(chain["decode_steps"]):
        arrays[f"chain_step{j}_input"] = f32(step["input"]).reshape(-1, H)
        arrays[f"chain_step{j}_output"] = f32(step["expected_output"]).reshape(-1)
        state_arrays(f"chain_step{j}_state", step["state"])
        steps.append({"length": step["state"]["length"],
                      "selection": selection_list(f"chain_step{j}", [step["selection"]])})
    sel_cases = []
    for j, c in enumerate(selv["cases"]):
        arrays[f"tier_{j}_scores"] = f32(c["selection"]["candidate_scores"]).reshape(-1)
        sel_cases.append({"id": c["id"], "mode": c["mode"], "limit": c["selection"]["selection_limit"],
                          "selected_block_ids": c["selection"]["selected_block_ids"],
                          "selected_token_positions": c["selection"]["selected_token_positions"],
                          "tail_positions": c["selection"]["tail_positions"]})
    meta = {"source": f"Kestrel-Q research/operators/Qwen3.8-Flash-Next/{REV}/qsa-*.json",
            "reduced_config": rc, "cases": cases, "chain_steps": steps, "selection_cases": sel_cases,
            "contracts": native["floating_contracts"], "selection_comparison": native["selection_comparison"]}
    np.savez_compressed(OUT / "qsa_golden.npz", **arrays)
    (OUT / "qsa_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


def moe(ops: Path) -> None:
    contract = json.loads((ops / "moe-contract.json").read_text())
    cal = json.loads((ops / "moe-calibration.json").read_text())
    hold = json.loads((ops / "moe-holdout.json").read_text())
    routing = json.loads((ops / "moe-routing-vectors.json").read_text())
    native = json.loads((ops / "moe-native-validation.json").read_text())
    tier = contract["tier_a_config"]
    E, H, I = tier["expert_count"], tier["hidden_size"], tier["routed_intermediate_size"]
    w = contract["weights"]
    arrays: dict[str, np.ndarray] = {}
    gate_up = f32(w["experts.gate_up_proj"]).reshape(E, 2 * I, H)   # gate rows, then up rows
    arrays["w_router"] = f32(w["gate.weight"]).reshape(-1)
    arrays["w_routed_gate"] = np.ascontiguousarray(gate_up[:, :I, :]).reshape(-1)
    arrays["w_routed_up"] = np.ascontiguousarray(gate_up[:, I:, :]).reshape(-1)
    arrays["w_routed_down"] = f32(w["experts.down_proj"]).reshape(-1)
    arrays["w_shared_gate"] = f32(w["shared_expert.gate_proj.weight"]).reshape(-1)
    arrays["w_shared_up"] = f32(w["shared_expert.up_proj.weight"]).reshape(-1)
    arrays["w_shared_down"] = f32(w["shared_expert.down_proj.weight"]).reshape(-1)
    arrays["w_shared_gate_weight"] = f32(w["shared_expert_gate.weight"]).reshape(-1)
    fields = ["final_output", "gated_shared_output", "routed_weighted_sum", "router_logits", "router_probabilities",
              "selected_weights", "shared_activated", "shared_gate", "shared_gate_logit", "shared_gate_projection",
              "shared_output", "shared_up_projection"]
    cases = []
    for split, src in (("calibration", cal["cases"]), ("holdout", hold["cases"])):
        for c in src:
            i = len(cases)
            x = f32(c["input"]).reshape(-1, H)
            arrays[f"c{i}_input"] = x
            for k in fields:
                arrays[f"c{i}_{k}"] = f32(c["expected"][k]).reshape(x.shape[0], -1)
            experts = []
            for j, e in enumerate(c["expected"]["selected_experts"]):
                for k in ("gate", "up", "activated", "output", "weighted_output"):
                    arrays[f"c{i}_e{j}_{k}"] = f32(e[k]).reshape(-1)
                experts.append({"token": e["token"], "expert_id": e["expert_id"],
                                "top_k_position": e["top_k_position"]})
            cases.append({"id": c["id"], "split": split, "selected_expert_ids": c["expected"]["selected_expert_ids"],
                          "selected_experts": experts})
    routing_cases = []
    for j, c in enumerate(routing["cases"]):
        arrays[f"r{j}_input"] = f32(c["input"]).reshape(-1, routing["config"]["hidden_size"])
        arrays[f"r{j}_router"] = f32(c["router_weight"]).reshape(-1)
        for k in ("router_logits", "router_probabilities", "selected_weights"):
            arrays[f"r{j}_{k}"] = f32(c["expected"][k]).reshape(arrays[f"r{j}_input"].shape[0], -1)
        routing_cases.append({"id": c["id"], "selected_expert_ids": c["expected"]["selected_expert_ids"]})
    contracts = {k: {kk: v[kk] for kk in ("class", "abs_limit", "rel_limit", "ulp_limit")}
                 for k, v in native["contracts"].items()}
    meta = {"source": f"Kestrel-Q research/operators/Qwen3.8-Flash-Next/{REV}/moe-*.json",
            "tier_a_config": tier, "tier_b_config": routing["config"], "routing_contract": contract["routing_contract"],
            "cases": cases, "routing_cases": routing_cases, "contracts": contracts,
            "comparison_classes": cal["comparison_classes"]}
    np.savez_compressed(OUT / "moe_golden.npz", **arrays)
    (OUT / "moe_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


def layer(ops: Path) -> None:
    """GDN and QSA decoder-layer cases (the PLE_GDN family needs the PLE
    operator, which the B200 library does not provide)."""
    cal = json.loads((ops / "layer-calibration.json").read_text())
    hold = json.loads((ops / "layer-holdout.json").read_text())
    contract = json.loads((ops / "layer-contract.json").read_text())
    native = json.loads((ops / "layer-native-validation.json").read_text())
    rc = contract["reduced"]
    H, B = rc["hidden"], rc["branches"]
    arrays: dict[str, np.ndarray] = {}
    gr = {"norm": "hc_norm.weight", "down": "input_mix_weight_down.weight", "up": "input_mix_weight_up.weight",
          "inject": "block_inject_weight.weight"}
    gdn_names = {"a_log": "A_log", "conv": "conv1d.weight", "dt_bias": "dt_bias", "alpha": "in_proj_a.weight",
                 "beta": "in_proj_b.weight", "qkv": "in_proj_qkv.weight", "gate": "in_proj_z.weight",
                 "norm": "norm.weight", "output": "out_proj.weight"}
    qsa_names = {"query": "q_proj.weight", "key": "k_proj.weight", "value": "v_proj.weight", "output": "o_proj.weight",
                 "query_norm": "q_norm.weight", "key_norm": "k_norm.weight",
                 "index_query_norm": "indexer.q_layernorm.weight", "index_key_norm": "indexer.k_layernorm.weight"}
    cases = []
    for split, src in (("calibration", cal["cases"]), ("holdout", hold["cases"])):
        for c in src:
            if c["family"] not in ("GDN", "QSA"):
                continue
            i = len(cases)
            w = c["weights"]
            T = c["input"]["shape"][1]
            arrays[f"c{i}_input"] = f32(c["input"]).reshape(T, B * H)
            arrays[f"c{i}_output"] = f32(c["output"]).reshape(T, B * H)
            for k, v in c["checkpoints"].items():
                arrays[f"c{i}_ck_{k}"] = f32(v).reshape(T, H)
            for side in ("attn", "mlp"):
                for k, v in gr.items():
                    arrays[f"c{i}_{side}_gr_{k}"] = f32(w[f"{side}_hyper_connection.{v}"]).reshape(-1)
            if c["family"] == "GDN":
                for k, v in gdn_names.items():
                    arrays[f"c{i}_gdn_{k}"] = f32(w[f"linear_attn.{v}"]).reshape(-1)
            else:
                for k, v in qsa_names.items():
                    arrays[f"c{i}_qsa_{k}"] = f32(w[f"self_attn.{v}"]).reshape(-1)
                qk = f32(w["self_attn.indexer.index_qk_proj.weight"])
                di = qk.shape[0] // 3   # index_qk rows: 2 query heads then the key head
                arrays[f"c{i}_qsa_index_query"] = qk[:2 * di].reshape(-1)
                arrays[f"c{i}_qsa_index_key"] = qk[2 * di:].reshape(-1)
            E = rc["experts"]
            I = rc["intermediate"]
            gate_up = f32(w["mlp.experts.gate_up_proj"]).reshape(E, 2 * I, H)
            arrays[f"c{i}_moe_router"] = f32(w["mlp.gate.weight"]).reshape(-1)
            arrays[f"c{i}_moe_routed_gate"] = np.ascontiguousarray(gate_up[:, :I, :]).reshape(-1)
            arrays[f"c{i}_moe_routed_up"] = np.ascontiguousarray(gate_up[:, I:, :]).reshape(-1)
            arrays[f"c{i}_moe_routed_down"] = f32(w["mlp.experts.down_proj"]).reshape(-1)
            arrays[f"c{i}_moe_shared_gate"] = f32(w["mlp.shared_expert.gate_proj.weight"]).reshape(-1)
            arrays[f"c{i}_moe_shared_up"] = f32(w["mlp.shared_expert.up_proj.weight"]).reshape(-1)
            arrays[f"c{i}_moe_shared_down"] = f32(w["mlp.shared_expert.down_proj.weight"]).reshape(-1)
            arrays[f"c{i}_moe_shared_gate_weight"] = f32(w["mlp.shared_expert_gate.weight"]).reshape(-1)
            cases.append({"id": c["id"], "split": split, "family": c["family"], "tokens": T,
                          "token_ids": c["token_ids"], "state_position": c["state_position"]})
    meta = {"source": f"Kestrel-Q research/operators/Qwen3.8-Flash-Next/{REV}/layer-*.json",
            "reduced": rc, "cases": cases, "validation": native["records"]}
    np.savez_compressed(OUT / "layer_golden.npz", **arrays)
    (OUT / "layer_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


def dequant(num: Path) -> None:
    d = json.loads((num / "dequant-vectors.json").read_text())
    keep = {"F32", "BF16", "Q8_0", "Q4_K"}
    cases = [{"id": c["id"], "type": c["type"], "packed_hex": c["packed_hex"],
              "expected_f32_bits": c["expected_f32_bits"], "pattern": c["pattern"]}
             for c in d["cases"] if c["type"] in keep]
    by_id = {c["id"]: c for c in d["cases"]}
    rows = [{"id": r["id"], "type": r["type"], "packed_hex": by_id[r["source_case_id"]]["packed_hex"],
             "activation_f32_bits": r["activation_f32_bits"], "expected_f32_bits": r["expected_f32_bits"]}
            for r in d["row_dot_cases"] if r["type"] in keep]
    meta = {"source": f"Kestrel-Q research/numerics/Qwen3.8-Flash-Next/{REV}/dequant-vectors.json",
            "oracle": d["oracle"], "comparison": "EXACT_BITS", "cases": cases, "row_dot_cases": rows}
    (OUT / "dequant_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    root = Path(a.reference) / "research"
    gdn(root / "operators" / "Qwen3.8-Flash-Next" / REV)
    qsa(root / "operators" / "Qwen3.8-Flash-Next" / REV)
    moe(root / "operators" / "Qwen3.8-Flash-Next" / REV)
    layer(root / "operators" / "Qwen3.8-Flash-Next" / REV)
    dequant(root / "numerics" / "Qwen3.8-Flash-Next" / REV)


if __name__ == "__main__":
    main()
