"""Synthetic-weight MLP latency benchmark on B200 (port of the reference's
bench/latency.py).

Same flags (--models, --sequence-lengths, --batch-size, --compress-ratio,
--benchmark {dense,xuv,gate-up,unfused,mlp,contracted-mlp,nki-parity,all},
--warmup, --iterations, --seed, --tuning-config, --output) and the same report
keys (bench/latency.py:96-126 timing keys, 269-314 per-result keys,
479-558 report and speed-up summary).  It imports the operators exactly as
the reference does, from ``svdflash_tpu.kernels.config`` and
``svdflash_tpu.kernels.pallas_ops``, which resolve to the sm_100a library.

B200 differences, each stated in the report:
  * every iteration is timed on the device with CUDA events and synchronised,
    the counterpart of perf_counter around jax.block_until_ready;
  * the factors are seeded torch draws with the reference's scales
    (N(0,1)/sqrt(rows)) instead of jax.random threefry draws;
  * "vendor" arms (the reference's XLA dots) run cuBLAS through torch.matmul;
    "unfused_svd_mlp" is the reference's six-matmul arm on the vendor GEMM and
    "unfused_svd_mlp_b200" the same six GEMMs on this library's svdmlp_gemm
    (test_speedup.py:690-736).
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
from collections.abc import Callable, Sequence

import torch

from svdflash_tpu.kernels.config import (
    MODELS,
    XUV_INPUT_TILE,
    XUV_OUTPUT_TILE,
    XUV_RANK_TILE,
    XUV_ROW_TILE,
    GateUpBlocks,
    fits_vmem,
    gate_up_block_params,
    rank_for,
    stage_plan,
    vmem_bytes_gate_up,
    vmem_bytes_gate_up_down_u,
    vmem_bytes_xuv,
)
from svdflash_tpu.kernels.pallas_ops import contracted_svd_mlp, dense_mlp, fused_gate_up, svd_mlp, xuv_matmul
from svdflash_tpu.test_speedup import unfused_low_rank, unfused_low_rank_pallas

BENCHMARKS = ("dense", "xuv", "gate-up", "unfused", "mlp", "contracted-mlp", "nki-parity", "all")


def _parse_sequence_lengths(value: str) -> tuple[int, ...]:
    lengths = tuple(int(item.strip()) for item in value.split(",") if item.strip())
    if not lengths or any(length <= 0 for length in lengths):
        raise argparse.ArgumentTypeError("sequence lengths must be positive integers")
    return lengths


def _random(gen: torch.Generator, shape, scale: float, device) -> torch.Tensor:
    return (torch.randn(*shape, generator=gen, device=device) * scale).to(torch.bfloat16)


def _make_factors(seed: int, hidden: int, intermediate: int, rank: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    hs, is_, rs = 1.0 / math.sqrt(hidden), 1.0 / math.sqrt(intermediate), 1.0 / math.sqrt(rank)
    return (_random(g, (hidden, rank), hs, device), _random(g, (rank, intermediate), rs, device),
            _random(g, (hidden, rank), hs, device), _random(g, (rank, intermediate), rs, device),
            _random(g, (intermediate, rank), is_, device), _random(g, (rank, hidden), rs, device))


def _make_dense_weights(seed: int, hidden: int, intermediate: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    hs, is_ = 1.0 / math.sqrt(hidden), 1.0 / math.sqrt(intermediate)
    return (_random(g, (hidden, intermediate), hs, device), _random(g, (hidden, intermediate), hs, device),
            _random(g, (intermediate, hidden), is_, device))


def _nearest_rank_percentile(samples: Sequence[float], percentile: float) -> float:
    index = min(len(samples) - 1, max(0, math.ceil(percentile / 100.0 * len(samples)) - 1))
    return samples[index]


def _measure(fn: Callable[..., torch.Tensor], args: Sequence[torch.Tensor], warmup: int,
             iterations: int) -> dict[str, float]:
    """Warm-up outside the measurement (the first call also packs the weights);
    then one device-timed, synchronised call per iteration."""
    for _ in range(warmup):
        fn(*args)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    samples_ms = []
    for _ in range(iterations):
        start.record()
        fn(*args)
        stop.record()
        stop.synchronize()
        samples_ms.append(start.elapsed_time(stop))
    samples_ms.sort()
    return {
        "latency_ms_avg": statistics.fmean(samples_ms),
        "latency_ms_p50": statistics.median(samples_ms),
        "latency_ms_p90": _nearest_rank_percentile(samples_ms, 90),
        "latency_ms_p95": _nearest_rank_percentile(samples_ms, 95),
        "latency_ms_p99": _nearest_rank_percentile(samples_ms, 99),
        "latency_ms_p100": samples_ms[-1],
        "latency_ms_min": samples_ms[0],
        "iterations": len(samples_ms),
        "measured_seconds": sum(samples_ms) / 1000.0,
    }


def _dense_vendor(x, w_gate, w_up, w_down):
    return (torch.nn.functional.silu(x @ w_gate) * (x @ w_up)) @ w_down


def _vendor_gate_up(x, u_gate, v_gate, u_up, v_up):
    return torch.nn.functional.silu((x @ u_gate) @ v_gate) * ((x @ u_up) @ v_up)


def _vendor_down_xuv(x, u_down, v_down):
    return (x @ u_down) @ v_down


def _load_tuned_blocks(path: str | None) -> dict:
    if path is None:
        return {}
    with open(path, "r", encoding="utf-8") as handle:
        report = json.load(handle)
    tuned = {}
    for record in report.get("best", []):
        if record["kernel"] != "gate-up":
            continue
        tuned[(record["model"], int(record["rows"]), "gate-up")] = (float(record["compress_ratio"]),
                                                                     GateUpBlocks(**record["blocks"]))
    return tuned


def _select_blocks(args, model_name: str, rows: int, kernel: str, default):
    entry = args.tuned_blocks.get((model_name, rows, kernel))
    if entry is None:
        return default
    tuned_ratio, blocks = entry
    if not math.isclose(tuned_ratio, args.compress_ratio, rel_tol=0.0, abs_tol=1e-9):
        raise ValueError(f"tuned {kernel} blocks for {model_name}, rows={rows} use compress_ratio={tuned_ratio}, "
                         f"requested {args.compress_ratio}")
    return blocks


def _timed(results, common, name, fn, fn_args, args, rows):
    timing = _measure(fn, fn_args, args.warmup, args.iterations)
    timing["throughput_tokens_per_second"] = rows * timing["iterations"] / timing["measured_seconds"]
    results.append({**common, "benchmark": name, **timing})


def _bench_model(args, model_name: str, device) -> list[dict]:
    model = MODELS[model_name]
    rank = rank_for(model, args.compress_ratio)
    hidden, inter = model.hidden_size, model.intermediate_size
    factors = dense_weights = None
    if args.benchmark in ("xuv", "gate-up", "unfused", "mlp", "contracted-mlp", "nki-parity", "all"):
        factors = _make_factors(args.seed, hidden, inter, rank, device)
    if args.benchmark in ("dense", "nki-parity", "all"):
        dense_weights = _make_dense_weights(args.seed + 10_000, hidden, inter, device)
    props = torch.cuda.get_device_properties(device)
    results = []
    for sequence_length in args.sequence_lengths:
        rows = args.batch_size * sequence_length
        g = torch.Generator(device=device)
        g.manual_seed(args.seed + rows)
        x = _random(g, (rows, hidden), 1.0, device)
        down_input = _random(g, (rows, inter), 1.0, device)
        gate_blocks = _select_blocks(args, model_name, rows, "gate-up",
                                     gate_up_block_params(rows, model, args.compress_ratio))
        contracted_blocks = gate_blocks._replace(bn=min(gate_blocks.bn, 512))
        gate_padded_rank = math.ceil(rank / gate_blocks.br) * gate_blocks.br
        contracted_padded_rank = math.ceil(rank / contracted_blocks.br) * contracted_blocks.br
        down_padded_rank = math.ceil(rank / XUV_RANK_TILE) * XUV_RANK_TILE
        gate_vmem = vmem_bytes_gate_up(gate_blocks, gate_padded_rank, hidden)
        down_vmem = vmem_bytes_xuv(inter, down_padded_rank, hidden)
        contracted_vmem = vmem_bytes_gate_up_down_u(contracted_blocks, contracted_padded_rank,
                                                    contracted_padded_rank, hidden)
        if not fits_vmem(gate_vmem) or not fits_vmem(down_vmem):
            raise ValueError(f"estimated SMEM exceeds the budget: gate/up={gate_vmem}, down={down_vmem}")
        gate_plan = stage_plan(1, rows, inter, rank)
        down_plan = stage_plan(2, rows, rank, inter)
        common = {
            "model": model_name,
            "batch_size": args.batch_size,
            "sequence_length": sequence_length,
            "rows": rows,
            "hidden_size": hidden,
            "intermediate_size": inter,
            "rank": rank,
            "logical_rank": rank,
            "compress_ratio": args.compress_ratio,
            "device": f"{props.name} (cuda:{device.index})",
            "gate_up_blocks": gate_blocks._asdict(),
            "contracted_blocks": contracted_blocks._asdict(),
            "down_tiles": {"rows": XUV_ROW_TILE, "input": XUV_INPUT_TILE, "rank": XUV_RANK_TILE,
                           "output": XUV_OUTPUT_TILE},
            "gate_up_padded_rank": gate_padded_rank,
            "down_padded_rank": down_padded_rank,
            "input_dtype": str(x.dtype).replace("torch.", ""),
            "scratch_dtype": "float16",
            "accumulator_dtype": "float32",
            "pallas_svd_dma_strategy": "tma_mbarrier_ring",
            "tensor_cores_per_device": props.multi_processor_count,
            "gate_up_row_tiles": math.ceil(rows / gate_blocks.bs),
            "down_row_tiles": math.ceil(rows / XUV_ROW_TILE),
            "active_tensor_cores_gate_up": min(props.multi_processor_count, gate_plan.grid),
            "active_tensor_cores_down": min(props.multi_processor_count, down_plan.grid),
            "estimated_gate_up_vmem_bytes": gate_vmem,
            "estimated_down_vmem_bytes": down_vmem,
            "estimated_contracted_vmem_bytes": contracted_vmem,
            "comparison_scope": "dense_vs_fused_low_rank_mlp" if args.benchmark == "nki-parity" else args.benchmark,
        }
        if args.benchmark in ("dense", "nki-parity", "all"):
            _timed(results, common, "dense_mlp", dense_mlp, (x, *dense_weights), args, rows)
            if args.benchmark == "all":
                _timed(results, common, "vendor_dense_mlp", _dense_vendor, (x, *dense_weights), args, rows)
        if args.benchmark in ("xuv", "all"):
            u_gate, v_gate, u_up, v_up, u_down, v_down = factors
            if args.benchmark == "all":
                _timed(results, common, "vendor_down_xuv", _vendor_down_xuv, (down_input, u_down, v_down), args,
                       rows)
            _timed(results, common, "down_xuv", lambda a, b, c: xuv_matmul(a, b, c), (down_input, u_down, v_down),
                   args, rows)
        if args.benchmark in ("gate-up", "all"):
            u_gate, v_gate, u_up, v_up, u_down, v_down = factors
            if args.benchmark == "all":
                _timed(results, common, "vendor_gate_up", _vendor_gate_up, (x, u_gate, v_gate, u_up, v_up), args,
                       rows)
            _timed(results, common, "fused_gate_up", lambda *xs: fused_gate_up(*xs, blocks=gate_blocks),
                   (x, u_gate, v_gate, u_up, v_up), args, rows)
        if args.benchmark in ("unfused", "all"):
            u_gate, v_gate, u_up, v_up, u_down, v_down = factors
            _timed(results, common, "unfused_svd_mlp",
                   lambda x_, ug, vg, uu, vu, ud, vd: unfused_low_rank(x_, uu, vu, ug, vg, ud, vd),
                   (x, *factors), args, rows)
            _timed(results, common, "unfused_svd_mlp_b200",
                   lambda x_, ug, vg, uu, vu, ud, vd: unfused_low_rank_pallas(x_, uu, vu, ug, vg, ud, vd),
                   (x, *factors), args, rows)
        if args.benchmark in ("mlp", "nki-parity", "all"):
            _timed(results, common, "two_kernel_svd_mlp", lambda *xs: svd_mlp(*xs, gate_up_blocks=gate_blocks),
                   (x, *factors), args, rows)
        if args.benchmark in ("contracted-mlp", "all"):
            _timed(results, common, "contracted_hidden_svd_mlp",
                   lambda *xs: contracted_svd_mlp(*xs, gate_up_blocks=contracted_blocks), (x, *factors), args,
                   rows)
        del x, down_input
    return results


def _parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--models", nargs="+", choices=tuple(MODELS), default=("qwen3-8b", "llama-3.1-8b"))
    parser.add_argument("--sequence-lengths", type=_parse_sequence_lengths, default=(1, 128, 512, 1024),
                        help="comma-separated token counts")
    parser.add_argument("--batch-size", type=int, default=1)
    parser.add_argument("--compress-ratio", type=float, default=0.8)
    parser.add_argument("--benchmark", choices=BENCHMARKS, default="all")
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--iterations", type=int, default=30)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--tuning-config", type=str, help="JSON written by a gate/up tuner run")
    parser.add_argument("--output", type=str)
    return parser


def _speedup_summary(results: Sequence[dict]) -> list[dict]:
    groups: dict = {}
    for result in results:
        groups.setdefault((result["model"], result["batch_size"], result["sequence_length"]), {})[
            result["benchmark"]] = result
    summaries = []
    for (model, batch_size, sequence_length), timings in groups.items():
        fused = timings.get("two_kernel_svd_mlp")
        contracted = timings.get("contracted_hidden_svd_mlp")
        if fused is None and contracted is None:
            continue
        summary = {"model": model, "batch_size": batch_size, "sequence_length": sequence_length}
        dense = timings.get("dense_mlp")
        unfused = timings.get("unfused_svd_mlp")
        unfused_b200 = timings.get("unfused_svd_mlp_b200")
        if fused is not None:
            summary["two_kernel_latency_ms"] = fused["latency_ms_avg"]
        if dense is not None and fused is not None:
            summary["speedup_vs_dense"] = dense["latency_ms_avg"] / fused["latency_ms_avg"]
        if unfused is not None and fused is not None:
            summary["speedup_vs_unfused_svd"] = unfused["latency_ms_avg"] / fused["latency_ms_avg"]
        if unfused_b200 is not None and fused is not None:
            summary["speedup_vs_unfused_svd_b200"] = unfused_b200["latency_ms_avg"] / fused["latency_ms_avg"]
        if contracted is not None:
            summary["contracted_hidden_latency_ms"] = contracted["latency_ms_avg"]
        if fused is not None and contracted is not None:
            summary["speedup_contracted_vs_two_kernel"] = fused["latency_ms_avg"] / contracted["latency_ms_avg"]
        if unfused is not None and contracted is not None:
            summary["speedup_contracted_vs_unfused_svd"] = unfused["latency_ms_avg"] / contracted["latency_ms_avg"]
        summaries.append(summary)
    return summaries


def main(argv=None) -> dict:
    args = _parser().parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("latency benchmark requires a CUDA device (B200)")
    if args.batch_size <= 0 or args.warmup < 0 or args.iterations <= 0:
        raise ValueError("batch-size and iterations must be positive; warmup may be zero")
    if not 0.0 < args.compress_ratio <= 1.0:
        raise ValueError("compress-ratio must be in the interval (0, 1]")
    args.tuned_blocks = _load_tuned_blocks(args.tuning_config)
    device = torch.device("cuda", torch.cuda.current_device())
    results = []
    for model_name in args.models:
        results.extend(_bench_model(args, model_name, device))
    report = {
        "synthetic_factors": True,
        "accuracy_claim": False,
        "benchmark_scope": "single_transformer_mlp_layer",
        "backend": "cuda",
        "jax_version": None,
        "torch_version": torch.__version__,
        "devices": [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())],
        "timing": "CUDA events per iteration, synchronised; same weights every iteration (as the reference)",
        "tuning_config": args.tuning_config,
        "tuned_workloads": len(args.tuned_blocks),
        "results": results,
        "speedups": _speedup_summary(results),
    }
    encoded = json.dumps(report, indent=2)
    print(encoded)
    if args.output:
        with open(args.output, "w", encoding="utf-8") as handle:
            handle.write(encoded + "\n")
    return report


if __name__ == "__main__":
    main()
