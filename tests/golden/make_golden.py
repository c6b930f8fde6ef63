"""Generate the golden vectors that pin the oracle to the reference.

Run in a container that has the mini-llm-runtime source tree (the reference
is pure Python + PyTorch; nothing here needs a GPU):

    python tests/golden/make_golden.py [--ref-src /path/to/mini-llm-runtime/src]

It imports the reference's own functions and writes seeded inputs together
with the reference's outputs to ``tests/golden/*.npz``:

* decode_config1.npz  — FP32 config 1 (B=4, Hq/Hkv 14/2, D 64, bs 16,
  contexts [17, 64, 100, 255], pool of 64 blocks, seeded randperm tables,
  one new token per sequence written through PagedKVCache.write_slots,
  unused slots filled with large finite values) -> paged_attention_decode_batch_parallel.
* decode_small.npz    — the cases of tests/kernels/test_paged_attention_batch.py.
* decode_bf16.npz     — config-1 geometry with BF16-representable values;
  the reference's FP32 path on the up-cast tensors (the BF16 parity target)
  and its own BF16 path.
* prefill_small.npz   — the grid of tests/kernels/test_paged_attention.py:249-351
  (MHA/GQA/MQA x prefix {0,5} x tile {1,4,16}, FP32, NaN-filled pools).
* prefill_medium.npz  — Hq/Hkv 14/2, D 64, bs 16, prefix 37, chunk 45 (FP32
  and BF16-valued), NaN-filled unused slots.
* write_slots.npz     — tests/runtime/test_write_slots_batch.py cases for
  FP32/FP16/BF16 pools from a non-contiguous FP32 source (bit patterns).
* accumulator.npz     — tests/kernels/test_accumulator_cuda.py expected value.
* runner_steps.npz    — three scheduler steps (whole prompts; a prompt with
  decodes; decodes) of the reference's TinyQwen2ForCausalLM through its
  build_model_batch and execute_model_batch (runtime/model_runner.py:37-272)
  on the seeded model and requests of tests/golden/runner_model.py: the
  ModelBatch tensors, packed logits, greedy tokens and the written KV rows.

The .npz files are committed; this script is how they were made.
"""

from __future__ import annotations

import argparse
import os
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def make_tables(ctx: list[int], num_blocks: int, bs: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    need = [(c + bs - 1) // bs for c in ctx]
    width = max(need)
    tables, cur = [], 0
    for n in need:
        row = perm[cur : cur + n]
        cur += n
        tables.append(row + [-1] * (width - n))
    return tables


def gen_decode_config1(ref):
    PagedKVCache = ref["PagedKVCache"]
    decode_parallel = ref["decode_parallel"]
    decode_reference = ref["decode_reference"]
    B, HQ, HKV, D, BS, NB = 4, 14, 2, 64, 16, 64
    ctx = [17, 64, 100, 255]
    tables = make_tables(ctx, NB, BS, seed=0)
    g = torch.Generator().manual_seed(1)
    cache = PagedKVCache(1, NB, BS, HKV, D, dtype=torch.float32, device="cpu")
    # Background (unused blocks / tail slots) is finite: the reference's
    # padded gather reads block 0 and tail slots for masked positions and
    # multiplies them by probability 0, so NaN there would poison its output
    # (paged_attention.py:232-235, :253).
    bg = torch.Generator().manual_seed(7)
    cache.k_cache.copy_(torch.randn(cache.k_cache.shape, generator=bg) * 100)
    cache.v_cache.copy_(torch.randn(cache.v_cache.shape, generator=bg) * 100)
    # Prior context (positions < ctx-1) is resident; the new token is written
    # through write_slots before attention, like forward_decode_batch_with_cache.
    for b in range(B):
        for pos in range(ctx[b] - 1):
            blk, off = tables[b][pos // BS], pos % BS
            cache.k_cache[0, blk, off] = torch.randn(HKV, D, generator=g)
            cache.v_cache[0, blk, off] = torch.randn(HKV, D, generator=g)
    k_pool0 = cache.k_cache.clone()
    v_pool0 = cache.v_cache.clone()
    q = torch.randn(B, HQ, D, generator=g)
    new_k = torch.randn(B, HKV, D, generator=g)
    new_v = torch.randn(B, HKV, D, generator=g)
    slots = torch.tensor([tables[b][(ctx[b] - 1) // BS] * BS + (ctx[b] - 1) % BS for b in range(B)])
    cache.write_slots(slots, new_k, new_v, layer_idx=0)
    kc, vc = cache.get_layer_cache(0)
    bt = torch.tensor(tables)
    cl = torch.tensor(ctx)
    out = decode_parallel(q, kc, vc, bt, cl, BS)
    out_ref = decode_reference(q, kc, vc, [t[: (c + BS - 1) // BS] for t, c in zip(tables, ctx)], ctx, BS)
    assert torch.isfinite(out).all()
    np.savez_compressed(
        HERE / "decode_config1.npz",
        old_k_at_slots=k_pool0.flatten(1, 2)[0, slots].numpy(),
        old_v_at_slots=v_pool0.flatten(1, 2)[0, slots].numpy(),
        k_pool=cache.k_cache.numpy(),
        v_pool=cache.v_cache.numpy(),
        q=q.numpy(),
        new_k=new_k.numpy(),
        new_v=new_v.numpy(),
        slot_mapping=slots.numpy(),
        block_tables=bt.numpy(),
        context_lens=cl.numpy(),
        block_size=np.int64(BS),
        out=out.numpy(),
        out_request_reference=out_ref.numpy(),
    )


def gen_decode_small(ref):
    decode_parallel = ref["decode_parallel"]
    cases = [
        (4, 2, [3, 5], [[2, 0, -1], [1, 3, 4]]),
        (2, 2, [3, 5], [[2, 0, -1], [1, 3, 4]]),
        (4, 1, [3, 5], [[2, 0, -1], [1, 3, 4]]),
        (4, 2, [3, 4], [[2, 0], [1, 3]]),
    ]
    arrays = {}
    for i, (hq, hkv, lens, tables) in enumerate(cases):
        torch.manual_seed(42)
        q = torch.randn(len(lens), hq, 8)
        k_cache = torch.randn(5, 2, hkv, 8)
        v_cache = torch.randn_like(k_cache)
        out = decode_parallel(q, k_cache, v_cache, torch.tensor(tables), torch.tensor(lens), 2)
        arrays.update(
            {
                f"c{i}_q": q.numpy(),
                f"c{i}_k": k_cache.numpy(),
                f"c{i}_v": v_cache.numpy(),
                f"c{i}_tables": np.array(tables, dtype=np.int64),
                f"c{i}_lens": np.array(lens, dtype=np.int64),
                f"c{i}_out": out.numpy(),
            }
        )
    arrays["num_cases"] = np.int64(len(cases))
    arrays["block_size"] = np.int64(2)
    np.savez_compressed(HERE / "decode_small.npz", **arrays)


def gen_decode_bf16(ref):
    decode_parallel = ref["decode_parallel"]
    B, HQ, HKV, D, BS, NB = 4, 14, 2, 64, 16, 64
    ctx = [17, 64, 100, 255]
    tables = make_tables(ctx, NB, BS, seed=0)
    g = torch.Generator().manual_seed(2)
    bg = torch.Generator().manual_seed(8)
    k = torch.randn((NB, BS, HKV, D), generator=bg) * 100
    v = torch.randn((NB, BS, HKV, D), generator=bg) * 100
    for b in range(B):
        for pos in range(ctx[b]):
            blk, off = tables[b][pos // BS], pos % BS
            k[blk, off] = torch.randn(HKV, D, generator=g)
            v[blk, off] = torch.randn(HKV, D, generator=g)
    q = torch.randn(B, HQ, D, generator=g)
    kb, vb, qb = k.bfloat16(), v.bfloat16(), q.bfloat16()
    bt, cl = torch.tensor(tables), torch.tensor(ctx)
    out32 = decode_parallel(qb.float(), kb.float(), vb.float(), bt, cl, BS)
    outbf = decode_parallel(qb, kb, vb, bt, cl, BS)
    np.savez_compressed(
        HERE / "decode_bf16.npz",
        k_pool_bits=_bits(kb),
        v_pool_bits=_bits(vb),
        q_bits=_bits(qb),
        block_tables=bt.numpy(),
        context_lens=cl.numpy(),
        block_size=np.int64(BS),
        out_fp32_reference=out32.numpy(),
        out_bf16_reference_bits=_bits(outbf),
    )


def _fill_paged(context_len, hkv, d, bs, block_table, dtype, gen):
    nb = max(block_table) + 1
    k_cache = torch.full((nb, bs, hkv, d), float("nan"), dtype=dtype)
    v_cache = torch.full_like(k_cache, float("nan"))
    lk = torch.randn(context_len, hkv, d, generator=gen).to(dtype)
    lv = torch.randn(context_len, hkv, d, generator=gen).to(dtype)
    for pos in range(context_len):
        k_cache[block_table[pos // bs], pos % bs] = lk[pos]
        v_cache[block_table[pos // bs], pos % bs] = lv[pos]
    return k_cache, v_cache


def gen_prefill_small(ref):
    tiled = ref["prefill_tiled"]
    dense = ref["prefill_tiled_reference"]
    arrays = {}
    i = 0
    for hq, hkv in [(2, 2), (4, 2), (4, 1)]:
        for prefix in [0, 5]:
            for tile in [1, 4, 16]:
                torch.manual_seed(0)
                chunk, d, bs, table = 4, 8, 3, [2, 0, 3]
                ctx = prefix + chunk
                q = torch.randn(chunk, hq, d)
                lk = torch.randn(ctx, hkv, d)
                lv = torch.randn_like(lk)
                k_cache = torch.full((4, bs, hkv, d), float("nan"))
                v_cache = torch.full_like(k_cache, float("nan"))
                for pos in range(ctx):
                    k_cache[table[pos // bs], pos % bs] = lk[pos]
                    v_cache[table[pos // bs], pos % bs] = lv[pos]
                out = tiled(q, k_cache, v_cache, table, prefix, ctx, bs, tile)
                out_dense = dense(q, k_cache, v_cache, table, prefix, ctx, bs, tile)
                arrays.update(
                    {
                        f"c{i}_q": q.numpy(),
                        f"c{i}_k": k_cache.numpy(),
                        f"c{i}_v": v_cache.numpy(),
                        f"c{i}_table": np.array(table, dtype=np.int64),
                        f"c{i}_meta": np.array([prefix, ctx, bs, tile], dtype=np.int64),
                        f"c{i}_out": out.numpy(),
                        f"c{i}_out_dense": out_dense.numpy(),
                    }
                )
                i += 1
    arrays["num_cases"] = np.int64(i)
    np.savez_compressed(HERE / "prefill_small.npz", **arrays)


def gen_prefill_medium(ref):
    tiled = ref["prefill_tiled"]
    dense = ref["prefill_tiled_reference"]
    hq, hkv, d, bs, prefix, chunk = 14, 2, 64, 16, 37, 45
    ctx = prefix + chunk
    g = torch.Generator().manual_seed(3)
    nblk = (ctx + bs - 1) // bs
    table = torch.randperm(nblk + 3, generator=g)[:nblk].tolist()
    k_cache, v_cache = _fill_paged(ctx, hkv, d, bs, table, torch.float32, g)
    q = torch.randn(chunk, hq, d, generator=g)
    out = tiled(q, k_cache, v_cache, table, prefix, ctx, bs, 16)
    out_dense = dense(q, k_cache, v_cache, table, prefix, ctx, bs, 16)
    # BF16-valued variant: FP32 reference on the up-cast values.
    kb, vb, qb = k_cache.bfloat16(), v_cache.bfloat16(), q.bfloat16()
    out_b = dense(qb.float(), kb.float(), vb.float(), table, prefix, ctx, bs, 16)
    np.savez_compressed(
        HERE / "prefill_medium.npz",
        q=q.numpy(),
        k=k_cache.numpy(),
        v=v_cache.numpy(),
        table=np.array(table, dtype=np.int64),
        meta=np.array([prefix, ctx, bs], dtype=np.int64),
        out=out.numpy(),
        out_dense=out_dense.numpy(),
        q_bits=_bits(qb),
        k_bits=_bits(kb),
        v_bits=_bits(vb),
        out_bf16_inputs_fp32_reference=out_b.numpy(),
    )


def gen_write_slots(ref):
    PagedKVCache = ref["PagedKVCache"]
    arrays = {}
    slots = [11, 0, 7, 4, 2]
    for name, dtype in [("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)]:
        torch.manual_seed(42)
        cache = PagedKVCache(2, 3, 4, 2, 8, dtype=dtype, device="cpu")
        cache.k_cache.normal_()
        cache.v_cache.normal_()
        before_k, before_v = cache.k_cache.clone(), cache.v_cache.clone()
        k = torch.randn(len(slots), 8, 2).transpose(1, 2)  # non-contiguous FP32
        v = torch.randn_like(k)
        cache.write_slots(torch.tensor(slots, dtype=torch.int32), k, v, layer_idx=1)
        arrays.update(
            {
                f"{name}_before_k": _bits(before_k),
                f"{name}_before_v": _bits(before_v),
                f"{name}_k": k.contiguous().numpy(),
                f"{name}_v": v.contiguous().numpy(),
                f"{name}_after_k": _bits(cache.k_cache),
                f"{name}_after_v": _bits(cache.v_cache),
            }
        )
    arrays["slots"] = np.array(slots, dtype=np.int64)
    np.savez_compressed(HERE / "write_slots.npz", **arrays)


def gen_accumulator():
    g = torch.Generator().manual_seed(0)
    p = torch.randn(7, 64, generator=g)
    v = torch.randn(7, 64, 256, generator=g)
    expected = torch.sum(p[:, :, None] * v, dim=1)
    np.savez_compressed(HERE / "accumulator.npz", p=p.numpy(), v=v.numpy(), out=expected.numpy())


def gen_runner_steps(ref):
    sys.path.insert(0, str(HERE))
    import runner_model as M

    config = ref["TinyQwen2Config"](**M.CONFIG)
    model = ref["TinyQwen2ForCausalLM"](config)
    model.load_state_dict(M.weights(), strict=True)
    model.eval()
    cache = ref["PagedKVCache"](M.CONFIG["num_hidden_layers"], M.NUM_BLOCKS, M.BLOCK_SIZE,
                                M.CONFIG["num_key_value_heads"], M.CONFIG["hidden_size"] // M.CONFIG["num_attention_heads"],
                                dtype=torch.float32, device="cpu")
    prompts, tables = M.prompts(), M.block_tables()
    reqs = {}
    for rid in M.PROMPT_LENS:
        reqs[rid] = ref["Request"](request_id=rid, prompt_token_ids=prompts[rid], max_new_tokens=8, arrival_time=0.0)
        reqs[rid].block_table = list(tables[rid])
    arrays = {}
    for s, (pre, dec) in enumerate(M.STEPS):
        sched = {rid: (len(prompts[rid]) - reqs[rid].num_computed_tokens) for rid in pre}
        sched.update({rid: 1 for rid in dec})
        out = ref["SchedulerOutput"](prefill_requests=[reqs[r] for r in pre], decode_requests=[reqs[r] for r in dec],
                                     num_scheduled_tokens=sched)
        batch = ref["build_model_batch"](out, M.BLOCK_SIZE, "cpu")
        with torch.no_grad():
            logits = ref["execute_model_batch"](model, batch, cache)
        qsl = batch.query_start_loc.tolist()
        sampled = [int(logits[qsl[i + 1] - 1].argmax()) for i in range(len(batch.request_ids))]
        for name in ("input_token_ids", "positions", "query_start_loc", "context_lens", "block_tables",
                     "slot_mapping"):
            arrays[f"s{s}_{name}"] = getattr(batch, name).numpy()
        arrays[f"s{s}_request_ids"] = np.array(batch.request_ids)
        arrays[f"s{s}_logits"] = logits.numpy()
        arrays[f"s{s}_sampled"] = np.array(sampled, dtype=np.int64)
        for i, rid in enumerate(batch.request_ids):
            reqs[rid].num_computed_tokens += sched[rid]
            reqs[rid].output_token_ids.append(sampled[i])
    # The pool rows the steps wrote: [L, slots, Hkv, D] at the sorted written slots.
    written = np.unique(np.concatenate([arrays[f"s{s}_slot_mapping"] for s in range(len(M.STEPS))]))
    arrays["written_slots"] = written
    arrays["k_written"] = cache.k_cache.flatten(1, 2)[:, written].numpy()
    arrays["v_written"] = cache.v_cache.flatten(1, 2)[:, written].numpy()
    np.savez_compressed(HERE / "runner_steps.npz", **arrays)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("MINI_LLM_RUNTIME_SRC"),
                    help="src/ directory of a mini-llm-runtime checkout (or set MINI_LLM_RUNTIME_SRC)")
    ap.add_argument("--only", default=None, help="generate only this fixture (file stem)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("--ref-src (or MINI_LLM_RUNTIME_SRC) is required")
    sys.path.insert(0, args.ref_src)
    from mini_llm_runtime.kernels.reference import paged_attention as pa_ref
    from mini_llm_runtime.runtime.paged_kv_cache import PagedKVCache
    from mini_llm_runtime.model.qwen2 import TinyQwen2Config, TinyQwen2ForCausalLM
    from mini_llm_runtime.runtime.model_runner import build_model_batch, execute_model_batch
    from mini_llm_runtime.runtime.request import Request
    from mini_llm_runtime.runtime.scheduler import SchedulerOutput

    ref = {
        "PagedKVCache": PagedKVCache,
        "decode_parallel": pa_ref.paged_attention_decode_batch_parallel,
        "decode_reference": pa_ref.paged_attention_decode_batch_reference,
        "prefill_tiled": pa_ref.paged_attention_prefill_chunk_tiled,
        "prefill_tiled_reference": pa_ref.paged_attention_prefill_chunk_tiled_reference,
        "TinyQwen2Config": TinyQwen2Config,
        "TinyQwen2ForCausalLM": TinyQwen2ForCausalLM,
        "build_model_batch": build_model_batch,
        "execute_model_batch": execute_model_batch,
        "Request": Request,
        "SchedulerOutput": SchedulerOutput,
    }
    torch.set_num_threads(1)
    gens = {
        "decode_config1": lambda: gen_decode_config1(ref),
        "decode_small": lambda: gen_decode_small(ref),
        "decode_bf16": lambda: gen_decode_bf16(ref),
        "prefill_small": lambda: gen_prefill_small(ref),
        "prefill_medium": lambda: gen_prefill_medium(ref),
        "write_slots": lambda: gen_write_slots(ref),
        "accumulator": gen_accumulator,
        "runner_steps": lambda: gen_runner_steps(ref),
    }
    for name, gen in gens.items():
        if args.only in (None, name):
            gen()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
