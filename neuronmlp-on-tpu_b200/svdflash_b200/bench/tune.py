"""Gate/up tuner on B200 (port of the reference's bench/tune.py).

Same flags and report layout (``records``, ``best`` with ``kernel``,
``model``, ``rows``, ``compress_ratio`` and ``blocks``), so that its output
feeds ``latency.py --tuning-config`` as the reference's does.  Candidates come
from ``config.gate_up_tuning_candidates``: on B200 the tile shape is compiled
in and the tunable knob is the split-K count of the SwiGLU GEMM, which
``fused_gate_up(blocks=...)`` applies per call.  Failures (a launch error or a
result outside the error bound) are recorded as candidate results, as the
reference records compile/run failures (bench/tune.py:34-100).
"""
from __future__ import annotations

import argparse
import json
import math
import sys

import torch

from svdflash_tpu.kernels.config import MODELS, gate_up_tuning_candidates, rank_for, vmem_bytes_gate_up
from svdflash_tpu.kernels.pallas_ops import fused_gate_up

from .latency import _make_factors, _measure, _parse_sequence_lengths, _random


def _run_candidate(*, blocks, fn, fn_args, rows, rank, hidden_size, warmup, iterations, expected,
                   max_relative_l2_error) -> dict:
    padded_rank = math.ceil(rank / blocks.br) * blocks.br
    record = {"kernel": "gate-up", "blocks": blocks._asdict(), "padded_rank": padded_rank,
              "estimated_vmem_bytes": vmem_bytes_gate_up(blocks, padded_rank, hidden_size)}
    try:
        timing = _measure(fn, fn_args, warmup, iterations)
        timing["throughput_tokens_per_second"] = rows * timing["iterations"] / timing["measured_seconds"]
        record.update(timing)
        record["status"] = "ok"
        if expected is not None:
            diff = fn(*fn_args).float() - expected
            rel = float(torch.linalg.norm(diff) / torch.clamp(torch.linalg.norm(expected), min=1e-12))
            record["max_abs_error"] = float(diff.abs().max())
            record["relative_l2_error"] = rel
            if not math.isfinite(rel) or rel > max_relative_l2_error:
                record.update(status="incorrect",
                              error=f"relative L2 error {rel:.6g} exceeds {max_relative_l2_error:.6g}")
    except Exception as error:  # noqa: BLE001 - launch failures are candidate results
        record.update(status="failed", error_type=type(error).__name__, error=str(error)[:1000])
    return record


def _tune_model(args, model_name: str, device):
    model = MODELS[model_name]
    rank = rank_for(model, args.compress_ratio)
    u_gate, v_gate, u_up, v_up, _, _ = _make_factors(args.seed, model.hidden_size, model.intermediate_size, rank,
                                                     device)
    records, best = [], []
    for sequence_length in args.sequence_lengths:
        rows = args.batch_size * sequence_length
        g = torch.Generator(device=device)
        g.manual_seed(args.seed + rows)
        x = _random(g, (rows, model.hidden_size), 1.0, device)
        expected = None
        if args.verify:
            # fp32 unfused reference of the same bf16 inputs (cuBLAS)
            xf = x.float()
            expected = (torch.nn.functional.silu((xf @ u_gate.float()) @ v_gate.float())
                        * ((xf @ u_up.float()) @ v_up.float()))
        candidates = gate_up_tuning_candidates(rows, model, args.compress_ratio, args.profile)
        if args.max_candidates > 0:
            candidates = candidates[:args.max_candidates]
        print(f"Tuning {model_name} rows={rows} kernel=gate-up candidates={len(candidates)}", file=sys.stderr)
        kernel_records = []
        for index, blocks in enumerate(candidates, start=1):
            record = _run_candidate(
                blocks=blocks, fn=lambda *xs, b=blocks: fused_gate_up(*xs, blocks=b),
                fn_args=(x, u_gate, v_gate, u_up, v_up), rows=rows, rank=rank, hidden_size=model.hidden_size,
                warmup=args.warmup, iterations=args.iterations, expected=expected,
                max_relative_l2_error=args.max_relative_l2_error)
            record.update(model=model_name, batch_size=args.batch_size, sequence_length=sequence_length, rows=rows,
                          compress_ratio=args.compress_ratio, rank=rank, candidate_index=index)
            records.append(record)
            kernel_records.append(record)
            status = f"{record['latency_ms_avg']:.4f} ms" if record["status"] == "ok" else record.get(
                "error_type", record["status"])
            print(f"  [{index}/{len(candidates)}] {blocks}: {status}", file=sys.stderr)
        ok = [r for r in kernel_records if r["status"] == "ok"]
        if ok:
            best.append(min(ok, key=lambda r: r["latency_ms_avg"]))
    return records, best


def _parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--models", nargs="+", choices=tuple(MODELS), default=("qwen3-8b",))
    parser.add_argument("--sequence-lengths", type=_parse_sequence_lengths, default=(1, 128, 512, 1024),
                        help="comma-separated token counts")
    parser.add_argument("--batch-size", type=int, default=1)
    parser.add_argument("--compress-ratio", type=float, default=0.8)
    parser.add_argument("--kernel", choices=("gate-up",), default="gate-up")
    parser.add_argument("--profile", choices=("quick", "full"), default="quick")
    parser.add_argument("--max-candidates", type=int, default=0,
                        help="limit candidates per kernel/workload; zero means all")
    parser.add_argument("--warmup", type=int, default=2)
    parser.add_argument("--iterations", type=int, default=10)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--verify", action=argparse.BooleanOptionalAction, default=True,
                        help="compare every candidate with an unfused fp32 reference")
    parser.add_argument("--max-relative-l2-error", type=float, default=0.05)
    parser.add_argument("--keep-compiler-cache", action="store_true", help="accepted; nothing is compiled at run time")
    parser.add_argument("--output", type=str, required=True)
    return parser


def main(argv=None) -> dict:
    args = _parser().parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("gate/up tuning requires a CUDA device (B200)")
    if args.batch_size <= 0 or args.warmup < 0 or args.iterations <= 0:
        raise ValueError("batch-size and iterations must be positive; warmup may be zero")
    if args.max_candidates < 0:
        raise ValueError("max-candidates may not be negative")
    if args.max_relative_l2_error <= 0:
        raise ValueError("max-relative-l2-error must be positive")
    if not 0.0 < args.compress_ratio <= 1.0:
        raise ValueError("compress-ratio must be in the interval (0, 1]")
    device = torch.device("cuda", torch.cuda.current_device())
    records, best = [], []
    for model_name in args.models:
        r, b = _tune_model(args, model_name, device)
        records.extend(r)
        best.extend(b)
    report = {"backend": "cuda", "jax_version": None, "torch_version": torch.__version__,
              "devices": [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())],
              "profile": args.profile, "records": records, "best": best}
    encoded = json.dumps(report, indent=2)
    print(encoded)
    with open(args.output, "w", encoding="utf-8") as handle:
        handle.write(encoded + "\n")
    return report


if __name__ == "__main__":
    main()
