"""Extract the reference's own golden vectors into compact fixtures for the parity tests.

Run once in a container where the reference checkout is mounted (it is read-only there and absent on the GPU
hosts, so the tests read only what this script writes):

    python tests/golden/make_golden.py --reference <path to the theolivenbaum/laya checkout>

Sources (paths inside the reference project):
  * tests/StructuredDecisions.Tests/Fixtures/training-tiny/  — model.safetensors (fp32 tiny ModernBERT +
    decision head), encoder/config.json, batch.json (items and PyTorch logits), grads.safetensors,
    objective.json (RLCD loss with recorded draws).  Made by tools/dump_training_reference.py:37-142.
  * tests/StructuredDecisions.Tests/Fixtures/qwen35-tiny/reference-q8_0.safetensors — `matmul.w/x/y`, one Q8_0
    product computed by torch as ggml does (tools/dump_mica_reference.py:158-190).
  * tests/StructuredDecisions.Tests/Fixtures/qwen35-tiny/ — the tiny Qwen3.5 decoder (model.safetensors, bf16), its
    config.json and reference.json (150 input ids), reference.safetensors (every layer's mixer output and output,
    the final norm and the last position's logits from transformers in fp32, and in fp64) and
    reference-q8_0.safetensors (the same from transformers computing every product as ggml's Q8_0 does), checked by
    Qwen35ParityTests.cs:45-136.
The tensors are copied bit for bit (bf16 widened to fp32 exactly); nothing is recomputed here.
"""
import argparse
import json
import os

import numpy as np
import torch
from safetensors.torch import load_file

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    fx = os.path.join(args.reference, "tests", "StructuredDecisions.Tests", "Fixtures")

    tiny = os.path.join(fx, "training-tiny")
    model = {k: v.float().numpy() for k, v in load_file(os.path.join(tiny, "model.safetensors")).items()}
    np.savez(os.path.join(HERE, "training_tiny_model.npz"), **model)
    grads = {k: v.float().numpy() for k, v in load_file(os.path.join(tiny, "grads.safetensors")).items()}
    np.savez(os.path.join(HERE, "training_tiny_grads.npz"), **grads)
    with open(os.path.join(tiny, "encoder", "config.json")) as f:
        enc = json.load(f)
    with open(os.path.join(tiny, "rl_agent_config.json")) as f:
        agent = json.load(f)
    with open(os.path.join(tiny, "batch.json")) as f:
        batch = json.load(f)
    with open(os.path.join(tiny, "objective.json")) as f:
        objective = json.load(f)
    with open(os.path.join(HERE, "training_tiny.json"), "w") as f:
        json.dump({"encoder_config": enc, "agent_config": agent, "batch": batch, "objective": objective}, f)

    q8 = load_file(os.path.join(fx, "qwen35-tiny", "reference-q8_0.safetensors"))
    np.savez(os.path.join(HERE, "q8_matmul.npz"),
             w=q8["matmul.w"].float().numpy(),      # bf16 values, exactly widened
             x=q8["matmul.x"].float().numpy(),
             y=q8["matmul.y"].float().numpy())
    qt = os.path.join(fx, "qwen35-tiny")
    weights = {k: v.float().numpy() for k, v in load_file(os.path.join(qt, "model.safetensors")).items()}
    np.savez(os.path.join(HERE, "qwen35_tiny_model.npz"), **weights)
    ref = {k: v.float().numpy() for k, v in load_file(os.path.join(qt, "reference.safetensors")).items()}
    np.savez(os.path.join(HERE, "qwen35_tiny_reference.npz"), **ref)
    refq = {k: v.float().numpy() for k, v in q8.items() if not k.startswith("matmul.")}
    np.savez(os.path.join(HERE, "qwen35_tiny_reference_q8_0.npz"), **refq)
    with open(os.path.join(qt, "config.json")) as f:
        cfg = json.load(f)
    with open(os.path.join(qt, "reference.json")) as f:
        meta = json.load(f)
    with open(os.path.join(HERE, "qwen35_tiny.json"), "w") as f:
        json.dump({"config": cfg, "input_ids": meta["input_ids"]}, f)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    torch.set_num_threads(1)
    main()
