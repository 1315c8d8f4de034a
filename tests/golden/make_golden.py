"""Generate the golden fixtures by running the REFERENCE implementation.

This script imports the reference project's own ``BaselineTransformer``,
``generate_random_case`` and ``compare_outputs``
(torch_transformer_benchmark.py:204-317, 1182-1220, 1237-1304) from a
checkout given by ``--reference`` and records, per case:

* the case's config, model seed, input seed and padding ratio;
* a SHA-256 of the reference model's state_dict (pins the oracle's
  seeded weight initialisation and parameter names);
* a SHA-256 of the reference's input tensor (pins input generation);
* the reference's fp32 output;
* the reference ``compare_outputs`` verdict on a deliberately perturbed copy
  of that output (pins the accuracy rule itself).

It runs on the CPU only and needs the reference checkout, so it is run once
in the build container and its outputs are committed; the tests never import
the reference.

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import hashlib
import pathlib
import sys

import torch

HERE = pathlib.Path(__file__).resolve().parent

# (name, batch, seq, d_model, heads, ffn, layers, causal, model_seed,
#  input_seed, padding_ratio)
CASES = [
    # BASELINE config c1 exactly (official shape 3).
    ("c1", 4, 128, 128, 4, 128, 4, True, 1234, 1234, 0.0),
    # c2/c4 geometry on a short batch: weights do not depend on B.
    ("c2_b8", 8, 128, 128, 4, 128, 4, True, 1234, 1235, 0.0),
    ("c4_b2", 2, 128, 128, 16, 128, 4, True, 1234, 1234, 0.0),
    # c3 geometry (head_dim 256) on one sequence.
    ("c3_b1", 1, 128, 1024, 4, 1024, 4, True, 1234, 1234, 0.0),
    # c5 geometry (head_dim 64, 2 layers) on a 256-token prefix.
    ("c5_s256", 1, 256, 1024, 16, 1024, 2, True, 1234, 1234, 0.0),
    # Edge cases: ragged sequence length, single token, padding, non-causal.
    ("ragged_s37", 3, 37, 128, 4, 128, 2, True, 7, 8, 0.0),
    ("single_token", 2, 1, 128, 4, 128, 2, True, 7, 9, 0.0),
    ("padded_c1", 4, 128, 128, 4, 128, 4, True, 1234, 1234, 0.25),
    ("noncausal_small", 2, 16, 128, 4, 512, 2, False, 5, 6, 0.0),
]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().float().contiguous().numpy().tobytes()).hexdigest()


def state_sha(module: torch.nn.Module) -> str:
    digest = hashlib.sha256()
    for key, value in module.state_dict().items():
        digest.update(key.encode())
        digest.update(value.detach().float().contiguous().numpy().tobytes())
    return digest.hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch_transformer_benchmark as ttb  # the reference itself

    torch.set_num_threads(max(1, torch.get_num_threads()))
    out_dir = pathlib.Path(args.out)
    for (name, b, s, d, h, f, l, causal, mseed, iseed, pad) in CASES:
        cfg = ttb.TransformerConfig(b, s, d, h, f, l, causal)
        cfg.validate()
        torch.manual_seed(mseed)
        model = ttb.BaselineTransformer(cfg).eval()
        x, mask = ttb.generate_random_case(
            cfg, torch.device("cpu"), torch.float32, iseed, pad, 1.0
        )
        with torch.inference_mode():
            y = model(x, mask)
        # Perturb a fixed set of elements by amounts straddling the rule.
        gen = torch.Generator().manual_seed(99)
        pert = y.clone()
        flat = pert.view(-1)
        idx = torch.randperm(flat.numel(), generator=gen)[: min(64, flat.numel())]
        flat[idx] += torch.linspace(-0.01, 0.01, idx.numel())
        verdict = ttb.compare_outputs(y, pert, rtol=0.02, atol=0.002)
        record = {
            "name": name,
            "config": dict(batch_size=b, seq_len=s, d_model=d, num_heads=h,
                           ffn_dim=f, num_layers=l, causal=causal),
            "model_seed": mseed,
            "input_seed": iseed,
            "padding_ratio": pad,
            "state_sha256": state_sha(model),
            "input_sha256": sha(x),
            "mask": mask.clone(),
            "output": y.clone(),
            "perturb_index": idx.clone(),
            "perturb_failed": verdict.failed_elements,
            "perturb_max_abs": verdict.max_abs_error,
            "perturb_worst_index": tuple(verdict.worst_index),
            "reference_commit_file": "torch_transformer_benchmark.py",
        }
        torch.save(record, out_dir / f"{name}.pt")
        print(f"{name}: out={tuple(y.shape)} perturb_failed={verdict.failed_elements}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
