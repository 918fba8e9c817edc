"""Budget calculators (no training): wire bytes per round of one path under each
compression mode, and device memory of a path or of the fused executor.

    python -m opendipaco_b200.utils.budget bandwidth --params 150e6 --tokens 10e9 --uplink-mbps 20
    python -m opendipaco_b200.utils.budget vram --hidden 2048 --layers 8 8 --vocab 128256 --paths-per-gpu 4

The byte counts follow this framework's own payload formats (``schedule/compress.py``):
fp32 or bf16 tensors; int8 = one byte per value plus one fp32 scale per tensor; int4 =
half a byte per value plus one fp32 scale per 128-value group; top-k sparse = an int32
index plus the encoded value for each kept entry. Weights travel down in bf16 at best
(a keyframe delta lets them go lower). Only the shared parameters of a path are counted:
private modules travel about once and are amortised away. The same analysis of the
reference is ``examples/bandwidth_budget.py`` / ``examples/vram_budget.py`` (the
``inner_steps`` lever: sync traffic scales as 1 / inner_steps).
"""

from __future__ import annotations

import argparse
import json

INT4_GROUP = 128
VALUE_BYTES = {"none": 4.0, "bf16": 2.0, "int8": 1.0, "int4": 0.5 + 4.0 / INT4_GROUP}


def per_param_bytes(compress: str = "none", down: str = "full", density: float = 1.0) -> tuple[float, float]:
    """(down, up) wire bytes per shared parameter per round."""
    if compress not in VALUE_BYTES:
        raise ValueError(f"compress must be one of {sorted(VALUE_BYTES)}, got {compress!r}")
    if not 0.0 < density <= 1.0:
        raise ValueError("density must be in (0, 1]")
    val = VALUE_BYTES[compress]
    if down == "delta" and compress in ("int8", "int4"):
        down_b = val                          # a quantized delta against the worker's keyframe
    else:
        down_b = 4.0 if compress == "none" else 2.0   # weights never below bf16
    up_b = val if density >= 1.0 else density * (4.0 + val)
    return down_b, up_b


def bandwidth_table(*, params: float, tokens: float, batch: int, seq_len: int, inner_steps=(50, 100, 250, 500),
                    uplink_mbps: float = 20.0, modes=None) -> list[dict]:
    """Rounds, total bytes and uplink hours to train ``tokens`` on one path, for each
    (inner steps, compression) pair."""
    modes = modes or [("none", "full", 1.0), ("bf16", "full", 1.0), ("int8", "delta", 1.0), ("int4", "delta", 1.0),
                      ("int8", "delta", 0.1)]
    rows = []
    for h in inner_steps:
        rounds = tokens / (batch * seq_len * h)
        for compress, down, density in modes:
            d, u = per_param_bytes(compress, down, density)
            up_total = rounds * params * u
            rows.append({"inner_steps": h, "compress": compress, "down": down, "density": density,
                         "rounds": round(rounds, 1), "down_GB": round(rounds * params * d / 1e9, 2),
                         "up_GB": round(up_total / 1e9, 2),
                         "uplink_hours": round(up_total * 8 / (uplink_mbps * 1e6) / 3600, 2)})
    return rows


def vram_table(*, hidden: int, heads: int, kv_heads: int | None, ffn: int, layers, vocab: int, levels,
               batch: int, seq_len: int, paths_per_gpu: int = 1) -> dict:
    """Device bytes of one path trained module by module, and of the fused executor
    holding ``paths_per_gpu`` paths."""
    from ..config import BackboneConfig, DiPaCoConfig
    from ..train.memory import fused_breakdown, vram_breakdown

    bb = BackboneConfig(vocab_size=vocab, hidden_size=hidden, num_attention_heads=heads,
                        num_key_value_heads=kv_heads, intermediate_size=ffn, layers_per_level=list(layers),
                        max_position_embeddings=max(2048, seq_len))
    cfg = DiPaCoConfig(backbone=bb, level_sizes=list(levels), sequence_length=seq_len)
    out = {"module_executor": vram_breakdown(cfg, batch_size=batch, seq_len=seq_len),
           "module_executor_bf16_ckpt": vram_breakdown(cfg, batch_size=batch, seq_len=seq_len, autocast=True,
                                                       checkpoint=True, chunked_logits=True),
           "fused_executor": fused_breakdown(cfg, paths_per_gpu=paths_per_gpu, batch_size=batch, seq_len=seq_len)}
    return {k: {n: (round(v / 2 ** 30, 3) if n not in ("n_params", "n_private") else v) for n, v in d.items()}
            for k, d in out.items()}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    b = sub.add_parser("bandwidth", help="wire bytes and uplink time per compression mode")
    b.add_argument("--params", type=float, default=150e6)
    b.add_argument("--tokens", type=float, default=10e9)
    b.add_argument("--batch", type=int, default=16)
    b.add_argument("--seq-len", type=int, default=2048)
    b.add_argument("--uplink-mbps", type=float, default=20.0)
    v = sub.add_parser("vram", help="device memory (GiB) of one path and of the fused executor")
    v.add_argument("--hidden", type=int, default=384)
    v.add_argument("--heads", type=int, default=6)
    v.add_argument("--kv-heads", type=int, default=None)
    v.add_argument("--ffn", type=int, default=1024)
    v.add_argument("--layers", type=int, nargs="+", default=[2, 2])
    v.add_argument("--levels", type=int, nargs="+", default=[4, 4])
    v.add_argument("--vocab", type=int, default=32000)
    v.add_argument("--batch", type=int, default=24)
    v.add_argument("--seq-len", type=int, default=128)
    v.add_argument("--paths-per-gpu", type=int, default=16)
    a = ap.parse_args(argv)
    if a.cmd == "bandwidth":
        for row in bandwidth_table(params=a.params, tokens=a.tokens, batch=a.batch, seq_len=a.seq_len,
                                   uplink_mbps=a.uplink_mbps):
            print(json.dumps(row))
    else:
        print(json.dumps(vram_table(hidden=a.hidden, heads=a.heads, kv_heads=a.kv_heads, ffn=a.ffn, layers=a.layers,
                                    vocab=a.vocab, levels=a.levels, batch=a.batch, seq_len=a.seq_len,
                                    paths_per_gpu=a.paths_per_gpu), indent=1))


if __name__ == "__main__":
    main()
