"""Process bodies for the tensor-parallel tests (spawned; one per rank).

Kept out of the test module so that ``multiprocessing`` spawn can import
them by name.
"""
import os
import sys
import traceback

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def _load_jal():
    from conftest import load_package
    return load_package()


def row_col_parallel_worker(rank, world, port, out_q):
    """CPU, gloo: a column-parallel (gate rows) and a row-parallel (down
    input columns) projection of the oracle over this rank's shard, combined
    with all_gather / all_reduce, next to the unsharded projection."""
    try:
        import torch
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        jal = _load_jal()
        import oracle_py as oracle
        H, F = 512, 1536
        plan = jal.tp_plan(8, 2, F, 4096, rank, world)
        f0, fn = plan["f_lo"], plan["f_n"]
        x = jal.synth_normal(H, seed=71, name="tp.x")
        z = jal.synth_normal(F, seed=72, name="tp.z")
        # column parallel: rows [f0, f0 + fn) of an F x H matrix
        raw_g = jal.synth_matrix(jal.Q4_0, F, H, seed=73, name="tp.gate")
        full_g = oracle.RepackedWeight(raw_g, jal.Q4_0, F, H).project_batch(x, 1)[0]
        rb = H // 32 * 18
        part_g = oracle.RepackedWeight(raw_g[f0 * rb:(f0 + fn) * rb], jal.Q4_0, fn, H).project_batch(x, 1)[0]
        gathered = [torch.zeros(fn) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(part_g.copy()))
        col = torch.cat(gathered).numpy()
        # row parallel: input columns [f0, f0 + fn) of an H x F matrix
        raw_d = jal.synth_matrix(jal.Q4_0, H, F, seed=74, name="tp.down")
        full_d = oracle.RepackedWeight(raw_d, jal.Q4_0, H, F).project_batch(z, 1)[0]
        blocks = raw_d.reshape(H, F // 32, 18)[:, f0 // 32:(f0 + fn) // 32, :]
        part_d = oracle.RepackedWeight(np.ascontiguousarray(blocks).ravel(), jal.Q4_0, H, fn).project_batch(
            z[f0:f0 + fn], 1)[0]
        red = torch.from_numpy(part_d.copy())
        dist.all_reduce(red)
        row = red.numpy()
        dist.destroy_process_group()
        out_q.put((rank, None, (col, full_g, row, full_d)))
    except Exception:
        out_q.put((rank, traceback.format_exc(), None))


def gpu_tp_worker(rank, world, uid, spec_kwargs, seed, prompt, tokens, steps, exchange, out_q):
    """One GPU per rank: this rank's shard of a synthetic model, prefill, the
    given tokens teacher-forced (logits of every step), then greedy decode on
    the device.  exchange "nccl" forces the all-reduce decode step."""
    try:
        import torch
        if exchange == "nccl":
            os.environ["JAL_TP_NCCL"] = "1"
        else:
            os.environ.pop("JAL_TP_NCCL", None)
        torch.cuda.set_device(rank)
        jal = _load_jal()
        jal.set_device(rank)
        tp = jal.TensorParallel(uid, rank, world)
        spec = jal.SynthSpec(**spec_kwargs)
        buf = jal.synth_gguf(spec, seed)
        recipe = jal.LlamaRecipe.from_gguf(buf)
        cache = recipe.build_repack_cache(buf, device=rank, tp=tp)
        ctx = jal.ExecutionContext(recipe, cache, n_ctx=256, kv_dtype=jal.KV_F16, numerics=jal.NUMERICS_FAST)
        mode = ctx.tp_exchange()
        logits = [ctx.prefill_step(prompt, 0)]
        for t in tokens:
            logits.append(ctx.decode_step(int(t)))
        ctx2 = jal.ExecutionContext(recipe, cache, n_ctx=256, kv_dtype=jal.KV_F16, numerics=jal.NUMERICS_FAST)
        l0 = ctx2.prefill_step(prompt, 0)
        greedy = ctx2.decode_greedy(int(np.argmax(l0)), steps)
        pos = ctx2.position()
        del ctx, ctx2, cache
        torch.cuda.synchronize()
        out_q.put((rank, None, (np.stack(logits), np.asarray(greedy), pos, mode)))
    except Exception:
        out_q.put((rank, traceback.format_exc(), None))
