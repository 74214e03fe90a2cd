"""Test infrastructure: bodies of the multi-rank CPU (gloo) tests, run by
torch.multiprocessing.spawn from tests/test_tp_gloo.py.  Each rank swaps h3tp.ops for
the oracle-backed CPU stand-in and runs the product's host orchestration."""
import os
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "minimax-h3-2xt4_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _init(rank, world, port, timeout_s=60):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    import oracle_ops
    oracle_ops.install()
    return dist


def problem(world, M=37, kl=512, N=96, seed=5):
    rng = np.random.default_rng(seed)
    K = kl * world
    gate = rng.standard_normal((M, K)).astype(np.float32)
    gate[::5] *= 4
    up = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    ws = (rng.uniform(1e-3, 1e-2, N) / 512).astype(np.float32)
    X = rng.standard_normal((M, N)).astype(np.float16)
    G = rng.standard_normal((3, N)).astype(np.float32)
    labels = (np.arange(M) % 3).astype(np.int32)
    xs = [np.concatenate([gate[:, r * kl:(r + 1) * kl], up[:, r * kl:(r + 1) * kl]], 1).astype(np.float16)
          for r in range(world)]
    wr = [np.ascontiguousarray(w[:, r * kl:(r + 1) * kl]) for r in range(world)]
    return xs, wr, ws, X, G, labels


def fc2_case(rank, world, port, outdir, mode, transport, scaled, payload="fp16"):
    import torch
    try:
        dist = _init(rank, world, port)
        from h3tp import swiglu_quant
        xs, wr, ws, X, G, labels = problem(world, N=256 if payload == "int8_gather" else 96)
        res = torch.from_numpy(X.copy())
        out = swiglu_quant.row_linear(torch.from_numpy(xs[rank]), torch.from_numpy(wr[rank]),
                                      torch.from_numpy(ws), dist, mode=mode, scaled_transport=scaled,
                                      residual=res, gate=torch.from_numpy(G),
                                      labels=torch.from_numpy(labels), transport=transport,
                                      payload=payload)
        assert out.data_ptr() == res.data_ptr()
        np.save(os.path.join(outdir, f"r{rank}.npy"), res.numpy())
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        Path(outdir, f"err{rank}.txt").write_text(traceback.format_exc())
        raise


def oproj_case(rank, world, port, outdir, K=None):
    import torch
    try:
        dist = _init(rank, world, port)
        from h3tp.tp_dit import RowParallelLinearINT8
        from h3tp.h3_operator_policy import H3OperatorPolicy
        rng = np.random.default_rng(9)
        M, K, N = 29, K or 256 * world, 64
        x = rng.standard_normal((M, K)).astype(np.float16)
        w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = (rng.uniform(1e-3, 1e-2, (N, 1)) / 512).astype(np.float32)
        mod = RowParallelLinearINT8(K, N, rank, world, device="cpu")
        mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(s))
        mod.operator_policy = H3OperatorPolicy()
        mod.comm = dist
        kl = K // world
        y = mod(torch.from_numpy(x[:, rank * kl:(rank + 1) * kl].copy()))
        np.save(os.path.join(outdir, f"r{rank}.npy"), y.numpy())
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        Path(outdir, f"err{rank}.txt").write_text(traceback.format_exc())
        raise


def guard_case(rank, world, port, outdir):
    """Unsupported geometry must raise ValueError on every rank before any collective."""
    import torch
    dist = _init(rank, world, port, timeout_s=20)
    from h3tp import swiglu_quant
    x = torch.zeros((4, 2 * 300), dtype=torch.float16)   # 300 is not whole 256-groups
    w = torch.zeros((8, 300), dtype=torch.int8)
    try:
        swiglu_quant.row_linear(x, w, torch.ones(8), dist, mode="fused_stored")
        Path(outdir, f"r{rank}.txt").write_text("no error")
    except ValueError as e:
        Path(outdir, f"r{rank}.txt").write_text("ValueError: " + str(e))
    dist.barrier()   # both ranks still agree afterwards: nothing was left half-collected
    dist.destroy_process_group()


def dead_rank_case(rank, world, port, outdir):
    """Rank 1 fails between steps and never joins the collective; rank 0's collective
    must end with an error from the short process-group timeout, not hang."""
    import torch
    import time
    dist = _init(rank, world, port, timeout_s=5)
    from h3tp import swiglu_quant
    xs, wr, ws, X, G, labels = problem(world)
    if rank == 1:
        Path(outdir, "r1.txt").write_text("left")
        os._exit(0)
    t0 = time.time()
    try:
        swiglu_quant.row_linear(torch.from_numpy(xs[0]), torch.from_numpy(wr[0]), torch.from_numpy(ws),
                                dist, mode="fused_stored", residual=torch.from_numpy(X.copy()))
        Path(outdir, "r0.txt").write_text("completed")
    except Exception as e:  # gloo raises on timeout / peer loss
        Path(outdir, "r0.txt").write_text(f"error after {time.time() - t0:.1f}s: {type(e).__name__}")
    os._exit(0)
