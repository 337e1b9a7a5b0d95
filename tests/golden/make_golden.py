"""Generate the golden fixtures in this directory from the reference's own code.

Run from the repository root, pointing at a checkout of the reference (read
only; nothing is written there), either with --ref or MLXZ_REFERENCE:

    python tests/golden/make_golden.py --ref <path to the metazen11/mlxz checkout>

The reference (metazen11/mlxz) is pure Python over MLX, which is macOS/arm64
only and not installed here.  Its KV-cache sources only use a handful of MLX
calls (mx.zeros, slicing assignment, mx.concatenate, mx.repeat,
mx.fast.scaled_dot_product_attention, mx.array); this script installs a
torch-CPU stand-in for ``mlx.core`` (plus no-op ``structlog`` and the two
``mlx_lm.models.cache`` helpers ``trim_prompt_cache`` uses) and then imports
and runs the reference's unmodified files:

  src/mlxz/paged_attention/block_manager.py, paged_kv.py, attention.py
  src/mlxz/prefix_cache/hasher.py, memory.py, base.py

The stand-in SDPA computes softmax(q.K^T * scale).V in float64 and returns
float32 (MLX's own kernel, which returns the input dtype, cannot run here).
Inputs come from oracle.rng (integer-only, reproducible anywhere); each
fixture records the SHA-256 of its inputs so a generator drift is caught.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import random
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import rng  # noqa: E402


# ---------------------------------------------------------------------------
# torch-CPU stand-in for the MLX calls the reference's KV path makes
# ---------------------------------------------------------------------------

class _ArrayMeta(type):
    def __instancecheck__(cls, obj):  # isinstance(x, mx.array)
        return isinstance(obj, torch.Tensor)


class _Array(metaclass=_ArrayMeta):
    def __new__(cls, x, dtype=None):  # mx.array(x): an independent copy
        t = torch.as_tensor(x)
        return (t if dtype is None else t.to(dtype)).clone()


def _sdpa(q, k, v, *, scale, mask=None):
    assert mask is None
    s = torch.matmul(q.double(), k.double().transpose(-1, -2)) * scale
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v.double()).float()


def install_shims() -> None:
    mx = types.ModuleType("mlx.core")
    mx.float16, mx.bfloat16, mx.float32 = torch.float16, torch.bfloat16, torch.float32
    mx.Dtype = torch.dtype
    mx.array = _Array
    mx.zeros = lambda shape, dtype=torch.float32: torch.zeros(shape, dtype=dtype)
    mx.ones = lambda shape, dtype=torch.float32: torch.ones(shape, dtype=dtype)
    mx.zeros_like = torch.zeros_like
    mx.ones_like = torch.ones_like
    mx.concatenate = lambda xs, axis=0: torch.cat(list(xs), dim=axis)
    # MLX repeat has numpy.repeat semantics: each slice repeated consecutively.
    mx.repeat = lambda a, repeats, axis: torch.repeat_interleave(a, repeats, dim=axis)
    mx.softmax = lambda a, axis=-1: torch.softmax(a, dim=axis)
    mx.eval = lambda *a, **k: None
    mx.allclose = lambda a, b: torch.tensor(bool(torch.allclose(a.float(), b.float())))
    mx.fast = types.SimpleNamespace(scaled_dot_product_attention=_sdpa)
    mlx = types.ModuleType("mlx")
    mlx.__path__ = []
    mlx.core = mx
    nn = types.ModuleType("mlx.nn")
    mlx.nn = nn
    sys.modules.update({"mlx": mlx, "mlx.core": mx, "mlx.nn": nn})

    # mlx_lm.models.cache: the names the prefix cache imports.
    cache = types.ModuleType("mlx_lm.models.cache")

    class KVCache:  # only used for isinstance checks in cache_type_name
        pass

    class QuantizedKVCache:
        def __init__(self, group_size=64, bits=8):
            self.group_size, self.bits, self.offset, self.step = group_size, bits, 0, 256
            self.keys = self.values = None

        @property
        def state(self):
            return self.keys, self.values

        @state.setter
        def state(self, v):
            self.keys, self.values = v

    def trim_prompt_cache(cache_list, num_tokens):
        # Trim `num_tokens` from every layer when all layers are trimmable.
        if not all(c.is_trimmable() for c in cache_list) or num_tokens == 0:
            return 0
        return [c.trim(num_tokens) for c in cache_list][0]

    cache.KVCache, cache.QuantizedKVCache = KVCache, QuantizedKVCache
    cache.trim_prompt_cache = trim_prompt_cache
    cache.make_prompt_cache = lambda model, max_kv_size=None: [KVCache() for _ in model.layers]
    for name in ("mlx_lm", "mlx_lm.models"):
        m = types.ModuleType(name)
        m.__path__ = []
        sys.modules[name] = m
    sys.modules["mlx_lm.models.cache"] = cache

    sl = types.ModuleType("structlog")

    class _Log:
        def __getattr__(self, _):
            return lambda *a, **k: None

    sl.get_logger = lambda *a, **k: _Log()
    sys.modules["structlog"] = sl

    # mlxz.config needs pydantic_settings (absent); cache_utils only imports
    # KVConfig from it for a type annotation.
    cfg = types.ModuleType("mlxz.config")

    class KVConfig:
        def __init__(self, bits=8, group_size=64, quantized_kv_start=512):
            self.bits, self.group_size, self.quantized_kv_start = bits, group_size, quantized_kv_start

    cfg.KVConfig = KVConfig
    sys.modules["mlxz.config"] = cfg


def load_reference(ref: Path) -> types.SimpleNamespace:
    src = ref / "src"
    sys.path.insert(0, str(src))
    import mlxz.paged_attention.attention as attention  # noqa: E402
    import mlxz.paged_attention.block_manager as block_manager
    import mlxz.paged_attention.paged_kv as paged_kv
    import mlxz.prefix_cache.hasher as hasher
    import mlxz.prefix_cache.memory as memory
    for m in (attention, block_manager, paged_kv, hasher, memory):
        assert str(ref) in m.__file__, m.__file__
    return types.SimpleNamespace(attention=attention, bm=block_manager, paged_kv=paged_kv,
                                 hasher=hasher, memory=memory)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.contiguous().view(torch.uint8 if a.dtype != torch.bool else torch.bool).numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


_TORCH = {"f16": torch.float16, "bf16": torch.bfloat16}


def bits_to_torch(bits: np.ndarray, dtype: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(_TORCH[dtype])


# ---------------------------------------------------------------------------
# Scenario A: one layer of the 1B-shape paged round trip + decode attention.
# ---------------------------------------------------------------------------

def c1_inputs(ctx=(37, 128, 300, 511), H=8, D=64, Hq=32, n_blocks=256, bs=16, dtype="f16"):
    perm = rng.permutation(1, n_blocks)
    tables, used = [], 0
    for c in ctx:
        nb = (c + 1 + bs - 1) // bs
        tables.append([int(x) for x in perm[used:used + nb]])
        used += nb
    pre_k = [rng.normal(2, (H, c, D), dtype, stream=b) for b, c in enumerate(ctx)]
    pre_v = [rng.normal(2, (H, c, D), dtype, stream=100 + b) for b, c in enumerate(ctx)]
    new_k = [rng.normal(3, (H, 1, D), dtype, stream=b) for b in range(len(ctx))]
    new_v = [rng.normal(3, (H, 1, D), dtype, stream=100 + b) for b in range(len(ctx))]
    q = [rng.normal(4, (Hq, 1, D), dtype, stream=b) for b in range(len(ctx))]
    return dict(ctx=list(ctx), H=H, D=D, Hq=Hq, n_blocks=n_blocks, bs=bs, dtype=dtype,
                tables=tables, pre_k=pre_k, pre_v=pre_v, new_k=new_k, new_v=new_v, q=q)


def inputs_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for key in ("pre_k", "pre_v", "new_k", "new_v", "q"):
        for a in inp[key]:
            h.update(np.ascontiguousarray(a).tobytes())
    h.update(json.dumps(inp["tables"]).encode())
    return h.hexdigest()


def scenario_c1(ref) -> None:
    inp = c1_inputs()
    dt = _TORCH[inp["dtype"]]
    bm = ref.bm.BlockManager(total_blocks=inp["n_blocks"], block_size=inp["bs"])
    cache = ref.paged_kv.PagedKVCache(bm, inp["H"], inp["D"], dtype=dt)
    out = {"name": "c1_layer", "inputs_sha256": inputs_digest(inp),
           "config": {k: inp[k] for k in ("ctx", "H", "D", "Hq", "n_blocks", "bs", "dtype")},
           "tables": inp["tables"], "seqs": []}
    attn = []
    scale = 1.0 / 8.0
    for b, c in enumerate(inp["ctx"]):
        sid = f"seq{b}"
        # Random block assignment is injected directly (BlockManager pops in order).
        cache._block_tables[sid] = list(inp["tables"][b])
        cache._offsets[sid] = 0
        cache.append_kv(sid, bits_to_torch(inp["pre_k"][b], "f16")[None],
                        bits_to_torch(inp["pre_v"][b], "f16")[None])
    for b in range(len(inp["ctx"])):
        sid = f"seq{b}"
        cache.append_kv(sid, bits_to_torch(inp["new_k"][b], "f16")[None],
                        bits_to_torch(inp["new_v"][b], "f16")[None])
    for b in range(len(inp["ctx"])):
        sid = f"seq{b}"
        k, v = cache.get_kv(sid)
        o = ref.attention.paged_attention_forward(bits_to_torch(inp["q"][b], "f16")[None],
                                                  cache, sid, scale=scale)
        attn.append(o[0].numpy().astype(np.float32))  # (Hq, 1, D)
        out["seqs"].append({"offset": cache.get_offset(sid), "k_sha256": sha(k),
                            "v_sha256": sha(v), "shape": list(k.shape),
                            "block_table": cache.get_block_table(sid)})
    out["k_pool_sha256"] = sha(cache._key_pool)
    out["v_pool_sha256"] = sha(cache._value_pool)
    out["scale"] = scale
    np.save(HERE / "c1_layer_attn.npy", np.stack(attn))
    (HERE / "c1_layer.json").write_text(json.dumps(out, indent=1))


# ---------------------------------------------------------------------------
# Scenario B: BlockManager-driven appends (block growth, free, block reuse).
# ---------------------------------------------------------------------------

def scenario_bm_paged(ref) -> None:
    H, D, Hq, dtype, n_blocks, bs = 2, 64, 4, "bf16", 24, 16
    dt = _TORCH[dtype]
    bm = ref.bm.BlockManager(total_blocks=n_blocks, block_size=bs)
    cache = ref.paged_kv.PagedKVCache(bm, H, D, dtype=dt)
    ops = []
    stream = [0]

    def kv(n):
        stream[0] += 1
        return (rng.normal(11, (H, n, D), dtype, stream=stream[0]),
                rng.normal(12, (H, n, D), dtype, stream=stream[0]))

    script = [("alloc", "a", 1), ("append", "a", 5), ("alloc", "b", 2), ("append", "b", 40),
              ("append", "a", 17), ("free", "a", None), ("alloc", "c", 1), ("append", "c", 3),
              ("append", "b", 1), ("append", "c", 30), ("alloc", "d", 0), ("append", "d", 16),
              ("append", "d", 1)]
    digest = hashlib.sha256()
    for op, sid, n in script:
        rec = {"op": op, "seq": sid, "n": n}
        if op == "alloc":
            cache.allocate_sequence(sid, n)
        elif op == "free":
            cache.free_sequence(sid)
        else:
            k, v = kv(n)
            digest.update(k.tobytes())
            digest.update(v.tobytes())
            rec["k_stream"] = stream[0]
            cache.append_kv(sid, bits_to_torch(k, dtype)[None], bits_to_torch(v, dtype)[None])
        rec["tables"] = {s: cache.get_block_table(s) for s in sorted(cache._block_tables)}
        rec["offsets"] = {s: cache.get_offset(s) for s in sorted(cache._offsets)}
        rec["stats"] = cache.stats
        rec["k_pool_sha256"] = sha(cache._key_pool)
        rec["v_pool_sha256"] = sha(cache._value_pool)
        ops.append(rec)
    gathers, attn = {}, []
    for i, sid in enumerate(sorted(cache._block_tables)):
        k, v = cache.get_kv(sid)
        q = rng.normal(13, (Hq, 1, D), dtype, stream=i)
        digest.update(q.tobytes())
        o = ref.attention.paged_attention_forward(bits_to_torch(q, dtype)[None], cache, sid)
        attn.append(o[0].numpy().astype(np.float32))
        gathers[sid] = {"k_sha256": sha(k), "v_sha256": sha(v), "shape": list(k.shape),
                        "q_stream": i}
    out = {"name": "bm_paged", "config": {"H": H, "D": D, "Hq": Hq, "dtype": dtype,
                                          "n_blocks": n_blocks, "bs": bs},
           "seeds": {"k": 11, "v": 12, "q": 13}, "inputs_sha256": digest.hexdigest(),
           "ops": ops, "gathers": gathers, "attn_order": sorted(cache._block_tables)}
    np.save(HERE / "bm_paged_attn.npy", np.stack(attn))
    (HERE / "bm_paged.json").write_text(json.dumps(out, indent=1))


# ---------------------------------------------------------------------------
# Scenario C: BlockManager operation traces (state after every op).
# ---------------------------------------------------------------------------

def _bm_state(bm) -> dict:
    return {"free_list": list(bm._free_list),
            "refcounts": [bm.get_refcount(i) for i in range(bm.total_blocks)],
            "allocated": [list(x) for x in bm._debug_state()["allocated"]]}


def scenario_bm_traces(ref, n_traces=30, steps=50) -> None:
    traces = []
    for t in range(n_traces):
        r = random.Random(1000 + t)
        total = r.choice([1, 2, 4, 8, 16, 32])
        bm = ref.bm.BlockManager(total_blocks=total, block_size=16)
        held: list[int] = []
        recs = []
        for _ in range(steps):
            kind = r.choice(["allocate", "allocate", "free", "incref", "cow", "free_bad",
                             "incref_bad", "allocate_neg"])
            if kind == "allocate":
                args = [r.randint(0, total + 1)]
            elif kind == "allocate_neg":
                kind, args = "allocate", [-r.randint(1, 3)]
            elif kind in ("free", "incref"):
                args = [r.sample(held, min(len(held), r.randint(1, 3)))] if held else [[]]
            elif kind in ("free_bad", "incref_bad"):
                kind = kind[:-4]
                args = [[r.randrange(total) for _ in range(r.randint(1, 3))]]
            else:
                args = [r.choice(held) if held and r.random() < 0.8 else r.randrange(total)]
            try:
                res = getattr(bm, "copy_on_write" if kind == "cow" else kind)(*args)
                rec = {"op": kind, "args": args, "result": res}
                if kind == "allocate":
                    held.extend(res)
                elif kind == "cow" and res != args[0]:
                    held.append(res)
            except ref.bm.OutOfBlocksError as e:
                rec = {"op": kind, "args": args,
                       "raises": {"type": "OutOfBlocksError", "requested": e.requested,
                                  "available": e.available}}
            except ref.bm.DoubleFreeError as e:
                rec = {"op": kind, "args": args,
                       "raises": {"type": "DoubleFreeError", "block_idx": e.block_idx}}
            except ValueError as e:
                rec = {"op": kind, "args": args, "raises": {"type": "ValueError", "msg": str(e)}}
            held = [b for b in held if bm.get_refcount(b) > 0]
            rec["state"] = _bm_state(bm)
            recs.append(rec)
        traces.append({"total_blocks": total, "block_size": 16, "ops": recs})
    (HERE / "block_manager_traces.json").write_text(json.dumps(traces))


# ---------------------------------------------------------------------------
# Scenario D: prefix hasher digests.
# ---------------------------------------------------------------------------

def scenario_hasher(ref) -> None:
    cases = []
    r = random.Random(7)
    for bs in (1, 3, 8, 16):
        for n in (0, 1, 7, 8, 9, 33, 100):
            toks = [r.randint(-2**31, 2**31 - 1) if r.random() < 0.1 else r.randint(0, 128_000)
                    for _ in range(n)]
            h = ref.hasher.RollingPrefixHasher(bs).hash_chunks(toks)
            cases.append({"block_size": bs, "tokens": toks, "digests": [d.hex() for d in h]})
    (HERE / "hasher.json").write_text(json.dumps(cases))


# ---------------------------------------------------------------------------
# Scenario E: PrefixCacheMemory policy traces (store/lookup/LRU/stats).
# ---------------------------------------------------------------------------

class MockKVCache:
    """KVCache-like layer with .state and trim (as in the reference's tests)."""

    def __init__(self, seq_len: int, head_dim: int, fill: float) -> None:
        self._keys = torch.full((1, 1, seq_len, head_dim), fill, dtype=torch.float32)
        self._values = torch.full((1, 1, seq_len, head_dim), fill + 1, dtype=torch.float32)

    @property
    def state(self):
        return (self._keys, self._values)

    def is_trimmable(self):
        return True

    def trim(self, n):
        if n <= 0:
            return 0
        self._keys = self._keys[:, :, :-n, :]
        self._values = self._values[:, :, :-n, :]
        return n


def scenario_prefix_memory(ref) -> None:
    traces = []
    for t in range(25):
        r = random.Random(5000 + t)
        budget = r.choice([1, 600, 2_000, 8_000, 10_000_000])
        cache = ref.memory.PrefixCacheMemory(memory_budget_bytes=budget)
        keys_seen: list[list[int]] = []
        recs = []
        for _ in range(30):
            if r.random() < 0.45 or not keys_seen:
                n_chunks = r.randint(1, 6)
                key = [r.randint(0, 5) for _ in range(n_chunks)]
                if keys_seen and r.random() < 0.5:
                    base = r.choice(keys_seen)
                    key = base[: r.randint(1, len(base))] + key[: r.randint(0, 2)]
                bs = r.choice([1, 2, 4, 8])
                n_layers = r.randint(1, 3)
                seq_len = r.randint(1, 12)
                n_tokens = r.choice([None, seq_len])
                layers = [MockKVCache(seq_len, 4, float(len(recs))) for _ in range(n_layers)]
                hashes = tuple(bytes([x]) * 32 for x in key)
                cache.store_sync(hashes, layers, n_tokens=n_tokens, block_size=bs)
                keys_seen.append(key)
                rec = {"op": "store", "key": key, "block_size": bs, "n_layers": n_layers,
                       "seq_len": seq_len, "n_tokens": n_tokens, "fill": float(len(recs))}
            else:
                base = r.choice(keys_seen)
                key = base[: r.randint(1, len(base))] + [r.randint(0, 5)
                                                         for _ in range(r.randint(0, 2))]
                hashes = tuple(bytes([x]) * 32 for x in key)
                ctype = r.choice([None, None, "MockKVCache", "QuantizedKVCache"])
                n, states, ct = cache.lookup_sync(hashes, cache_type=ctype)
                rec = {"op": "lookup", "key": key, "cache_type": ctype, "n": n,
                       "result_type": ct, "hit": states is not None}
                if states is not None:
                    rec["state_len"] = int(states[0][0].shape[2])
                    rec["state_fill"] = float(states[0][0].flatten()[0]) if states[0][0].numel() else None
                    rec["n_layers"] = len(states)
            st = cache.stats()
            rec["stats"] = {"hits": st.hits, "misses": st.misses, "hit_bytes": st.hit_bytes,
                            "evictions": st.evictions, "memory_used_bytes": st.memory_used_bytes}
            rec["entries"] = sorted([[h[0] for h in k] for k in cache._entries])
            recs.append(rec)
        traces.append({"budget": budget, "ops": recs})
    (HERE / "prefix_memory_traces.json").write_text(json.dumps(traces))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MLXZ_REFERENCE"),
                    help="path of the reference checkout (default: $MLXZ_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or MLXZ_REFERENCE")
    install_shims()
    ref = load_reference(Path(a.ref))
    scenario_c1(ref)
    scenario_bm_paged(ref)
    scenario_bm_traces(ref)
    scenario_hasher(ref)
    scenario_prefix_memory(ref)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
