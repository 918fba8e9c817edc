"""Test-time routing and evaluation (reference ``src/opendipaco/inference.py:27-173``).

* ``compose_path`` aliases the trained bank (no copy).
* ``perplexity``: exp of the mean of per-batch mean losses.
* ``routed_perplexity``: route each sequence by its first ``prefix_len`` tokens,
  score only targets at positions >= prefix_len (the paper's protocol), token-level
  sum / count, exp.
* ``routed_window_perplexity``: re-route every ``window`` tokens from the previous
  window and score each window under its path with the full preceding context, the
  reference's definition. By default the context is not recomputed: each (sequence,
  path) pair keeps the per-layer keys and values of the tokens it has processed and
  only extends them, so every token passes each path at most once instead of once per
  later window (``kv_cache=False`` recomputes the prefix like the reference).

On CUDA ``routed_perplexity`` scores the routed sequences of up to 16 paths side by
side (``GroupedScorer``: one grouped forward with the training step's tcgen05 kernels,
LM head in row chunks, per-row CE kernel); otherwise, and for a custom ``compose_fn``,
each path's batches run through its module forward and the per-row CE kernel (no
[tokens, vocab] fp32 logits copy).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from .config import DiPaCoConfig
from .models.llama import apply_rope, rope_cos_sin
from .models.path import PathModel, build_path_model
from .routing.base import Featurizer, Router
from .topology import Path


def compose_path(config: DiPaCoConfig, bank: dict[str, nn.Module], path: Path) -> PathModel:
    return build_path_model(config, path, bank, deepcopy=False)


def route(prefixes: list[torch.Tensor], router: Router, featurizer: Featurizer) -> torch.Tensor:
    return router.predict(featurizer(prefixes))


def _ce_sum(pred: torch.Tensor, tgt: torch.Tensor) -> float:
    if pred.is_cuda:
        from .ops import loss as L

        return float(L.cross_entropy_sum(pred.reshape(-1, pred.size(-1)), tgt.reshape(-1)))
    return float(F.cross_entropy(pred.reshape(-1, pred.size(-1)), tgt.reshape(-1), reduction="sum"))


@torch.no_grad()
def perplexity(model: PathModel, sequences: torch.Tensor, batch_size: int = 8) -> float:
    model.eval()
    dev = next(model.parameters()).device
    total, n = 0.0, 0
    for i in range(0, sequences.size(0), batch_size):
        batch = sequences[i:i + batch_size].to(dev)
        _, loss = model(batch, labels=batch)
        total += float(loss)
        n += 1
    return float("nan") if n == 0 else float(torch.exp(torch.tensor(total / n)))


def config_path(config: DiPaCoConfig, path_index: int) -> Path:
    return config.build_topology().path_from_index(path_index)


@torch.no_grad()
def routed_perplexity(config: DiPaCoConfig, bank: dict[str, nn.Module], sequences: torch.Tensor,
                      router: Router, featurizer: Featurizer, prefix_len: int = 32,
                      batch_size: int = 8, compose_fn=None) -> float:
    paths = route([s[:prefix_len] for s in sequences], router, featurizer)
    start = max(prefix_len, 1)
    if compose_fn is None and sequences.numel() and sequences.size(1) > start:
        from .train.scorer import GroupedScorer

        dev = next(next(iter(bank.values())).parameters()).device
        if GroupedScorer.supported(config, dev):
            return _grouped_routed_perplexity(config, bank, sequences, paths, start, batch_size, dev)
    total, count = 0.0, 0
    for pidx in paths.unique().tolist():
        path = config_path(config, pidx)
        model = compose_fn(path) if compose_fn is not None else compose_path(config, bank, path)
        dev = next(model.parameters()).device
        seqs = sequences[paths == pidx]
        for i in range(0, seqs.size(0), batch_size):
            batch = seqs[i:i + batch_size].to(dev)
            if batch.size(1) <= start:
                continue
            logits, _ = model(batch)
            total += _ce_sum(logits[:, start - 1:-1, :], batch[:, start:])
            count += batch[:, start:].numel()
    return float("nan") if count == 0 else float(torch.exp(torch.tensor(total / count)))


def _grouped_routed_perplexity(config, bank, sequences, paths, start, batch_size, dev) -> float:
    """Token-level routed perplexity with the paths' batches scored side by side: a wave
    takes the next batch of up to ``batch_size`` sequences of up to G paths."""
    from .train.scorer import GroupedScorer, group_count, padded_len, shifted_targets

    tasks = []
    for pidx in paths.unique().tolist():
        rows = (paths == pidx).nonzero(as_tuple=True)[0]
        tasks += [(pidx, rows[i:i + batch_size]) for i in range(0, rows.numel(), batch_size)]
    n, slen = sequences.shape
    G = group_count(config, bank, min(16, len(tasks)))
    B = min(batch_size, n)
    S = padded_len(slen)
    sc = GroupedScorer(config, bank, dev, G, B, S)
    topo = config.build_topology()
    total = torch.zeros((), dtype=torch.float64)
    count = 0
    for w0 in range(0, len(tasks), G):
        wave = tasks[w0:w0 + G]
        ids = torch.zeros(G, B, S, dtype=torch.long)
        valid = torch.zeros(G, B, S, dtype=torch.bool)
        for g in range(G):
            pidx, rows = wave[g] if g < len(wave) else wave[0]
            sc.load(g, topo.path_from_index(pidx))
            if g < len(wave):
                ids[g, :rows.numel(), :slen] = sequences[rows]
                valid[g, :rows.numel(), :slen] = True
                count += rows.numel() * (slen - start)
        ids, valid = ids.to(dev), valid.to(dev)
        tgt = shifted_targets(ids.view(G * B, S), valid.view(G * B, S), first=start).view(G, B, S)
        total += sc.token_losses(ids, tgt).double().sum().cpu()
    return float("nan") if count == 0 else float(torch.exp(total / count))


def _norm(mod, x: torch.Tensor) -> torch.Tensor:
    h = x.float()
    return mod.weight * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + mod.variance_epsilon))


def _extend(model: PathModel, ids: torch.Tensor, cache: list | None, start: int):
    """Run tokens ``ids`` [b, n] at positions ``start, start + 1, ...`` through ``model``
    given each layer's cached (keys, values) of positions ``< start``; returns the
    logits [b, n, vocab] and the extended cache. Plain fp32 tensor ops on any device
    (the same arithmetic as the modules' reference forward)."""
    bb = model.config.backbone
    x = F.embedding(ids, model.embed.embed_tokens.weight).float()
    b, n = ids.shape
    cos, sin = rope_cos_sin(bb.head_dim, bb.rope_theta, n, ids.device, offset=start)
    layers = [layer for block in model.body for layer in block.layers]
    out = []
    for i, layer in enumerate(layers):
        att = layer.self_attn
        h = _norm(layer.input_layernorm, x)
        q = F.linear(h, att.q_proj.weight).view(b, n, att.num_heads, att.head_dim).transpose(1, 2)
        k = F.linear(h, att.k_proj.weight).view(b, n, att.num_kv, att.head_dim).transpose(1, 2)
        v = F.linear(h, att.v_proj.weight).view(b, n, att.num_kv, att.head_dim).transpose(1, 2)
        q, k = apply_rope(q, cos, sin).to(v.dtype), apply_rope(k, cos, sin).to(v.dtype)
        if cache is not None:
            k, v = torch.cat([cache[i][0], k], dim=2), torch.cat([cache[i][1], v], dim=2)
        out.append((k, v))
        if att.num_kv != att.num_heads:
            rep = att.num_heads // att.num_kv
            k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        total = k.shape[2]
        mask = torch.ones(n, total, dtype=torch.bool, device=ids.device).tril(diagonal=total - n)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        x = x + F.linear(o.transpose(1, 2).reshape(b, n, att.num_heads * att.head_dim), att.o_proj.weight)
        h = _norm(layer.post_attention_layernorm, x)
        mlp = layer.mlp
        x = x + F.linear(F.silu(F.linear(h, mlp.gate_proj.weight)) * F.linear(h, mlp.up_proj.weight),
                         mlp.down_proj.weight)
    return F.linear(_norm(model.head.norm, x), model.head.lm_head.weight), out


def _cached_windows(models, route_window, sequences, window, prefix_len, batch_size, dev):
    """Token-level (CE sum, count) of the windowed protocol with per-(sequence, path)
    key/value caches; a cache is cut back to the position whose logits score the
    window's first target before it is extended."""
    nseq, slen = sequences.shape
    caches: dict = {}  # (sequence, path) -> (cached length, [(k, v)] per layer, each [1, kv, len, d])
    total, count = 0.0, 0
    for w in range(math.ceil(slen / window)):
        w0, w1 = w * window, min((w + 1) * window, slen)
        t0 = max(w0, prefix_len, 1)
        if t0 >= w1:
            continue
        paths = route_window(w)
        for pidx in paths.unique().tolist():
            model = models(pidx)
            rows = (paths == pidx).nonzero(as_tuple=True)[0].tolist()
            by_start: dict = {}
            for r in rows:  # resume each sequence from what its cache under this path holds
                c = min(caches.get((r, pidx), (0, None))[0], t0 - 1)
                by_start.setdefault(c, []).append(r)
            for c, rs in sorted(by_start.items()):
                for s0 in range(0, len(rs), batch_size):
                    part = rs[s0:s0 + batch_size]
                    ids = sequences[part, c:w1].to(dev)
                    cache = None
                    if c > 0:
                        per = [caches[(r, pidx)][1] for r in part]
                        cache = [(torch.cat([p[i][0][:, :, :c] for p in per]),
                                  torch.cat([p[i][1][:, :, :c] for p in per])) for i in range(len(per[0]))]
                    logits, new = _extend(model, ids, cache, c)
                    for j, r in enumerate(part):
                        caches[(r, pidx)] = (w1, [(k[j:j + 1], v[j:j + 1]) for k, v in new])
                    total += _ce_sum(logits[:, t0 - 1 - c:w1 - 1 - c, :], ids[:, t0 - c:])
                    count += len(part) * (w1 - t0)
    return total, count


@torch.no_grad()
def routed_window_perplexity(config: DiPaCoConfig, bank: dict[str, nn.Module],
                             sequences: torch.Tensor, router: Router, featurizer: Featurizer,
                             window: int = 64, batch_size: int = 8, compose_fn=None,
                             prefix_len: int = 32, kv_cache: bool = True) -> float:
    if sequences.numel() == 0:
        return float("nan")
    if kv_cache:
        dev = next(next(iter(bank.values())).parameters()).device
        topo = config.build_topology()
        nseq, slen = sequences.shape
        built: dict = {}

        def models(pidx):
            if pidx not in built:
                p = topo.path_from_index(pidx)
                built[pidx] = (compose_fn(p) if compose_fn is not None else compose_path(config, bank, p)).eval()
            return built[pidx]

        def route_window(w):
            rc = w - 1 if w > 0 else 0
            return route([sequences[n, rc * window:min((rc + 1) * window, slen)] for n in range(nseq)],
                         router, featurizer)

        total, count = _cached_windows(models, route_window, sequences, window, prefix_len, batch_size, dev)
        return float("nan") if count == 0 else float(torch.exp(torch.tensor(total / count)))
    dev = next(next(iter(bank.values())).parameters()).device
    topo = config.build_topology()
    nseq, slen = sequences.shape
    models: dict[int, PathModel] = {}
    total, count = 0.0, 0
    for w in range(math.ceil(slen / window)):
        w0, w1 = w * window, min((w + 1) * window, slen)
        t0 = max(w0, prefix_len, 1)
        if t0 >= w1:
            continue
        rc = w - 1 if w > 0 else 0
        paths = route([sequences[n, rc * window:min((rc + 1) * window, slen)] for n in range(nseq)],
                      router, featurizer)
        for pidx in paths.unique().tolist():
            rows = (paths == pidx).nonzero(as_tuple=True)[0]
            model = models.get(pidx)
            if model is None:
                p = topo.path_from_index(pidx)
                model = (compose_fn(p) if compose_fn is not None else compose_path(config, bank, p)).eval()
                models[pidx] = model
            for s in range(0, rows.numel(), batch_size):
                batch = sequences[rows[s:s + batch_size], :w1].to(dev)
                logits, _ = model(batch)
                total += _ce_sum(logits[:, t0 - 1:w1 - 1, :], batch[:, t0:w1])
                count += batch[:, t0:w1].numel()
    return float("nan") if count == 0 else float(torch.exp(torch.tensor(total / count)))
