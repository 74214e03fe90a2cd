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


def _full_block(H, heads, hd, F, T, seed=3):
    """A stand-in for the reference's full (unsharded) DiT block: the parameters
    TPDiTBlockINT8.load_from_full_block reads, under the names it reads them by."""
    import torch
    from torch import nn
    g = torch.Generator().manual_seed(seed)

    def proj(n, k, div=1.0):
        m = nn.Module()
        m.register_buffer("weight", torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8))
        m.register_buffer("weight_scale", (torch.rand((n, 1), generator=g) * 9e-3 + 1e-3) / div)
        return m

    def norm(n):
        m = nn.Module()
        m.weight = nn.Parameter(1.0 + 0.1 * torch.randn(n, generator=g))
        return m

    blk = nn.Module()
    blk.norm1, blk.norm2 = norm(H), norm(H)
    blk.attn = nn.Module()
    blk.attn.q_norm, blk.attn.k_norm = norm(hd), norm(hd)
    blk.attn.qkv_proj = proj(3 * heads * hd, H)
    blk.attn.out_proj = proj(H, heads * hd, 64.0)
    blk.mlp = nn.Module()
    blk.mlp.fc1 = proj(2 * F, H)
    blk.mlp.fc2 = proj(H, F, 64.0)
    blk.adaln_proj = nn.Module()
    blk.adaln_proj.apply_silu = True
    blk.adaln_proj.linear = nn.Linear(T, 6 * 3 * H)
    with torch.no_grad():
        blk.adaln_proj.linear.weight.copy_(0.05 * torch.randn(6 * 3 * H, T, generator=g))
        blk.adaln_proj.linear.bias.copy_(0.05 * torch.randn(6 * 3 * H, generator=g))
    return blk


def reference_block_case(rank, world, port, outdir, refdir):
    """The reference's own TPDiTBlockINT8 (patches/tp_dit.py) with this library's
    projection modules swapped in as INTEGRATION.md shows: the block is built, loaded
    with load_from_full_block and run by the reference's code; only the four projections
    are ours (their kernels replaced by the oracle-backed stand-in on CPU ranks).
    `comfy_kitchen` is imported at the top of the reference module but used only by
    the RoPE branch, which this case does not take; an empty module stands in for it."""
    import types
    import torch
    try:
        dist = _init(rank, world, port)
        sys.modules.setdefault("comfy_kitchen", types.ModuleType("comfy_kitchen"))
        if refdir not in sys.path:
            sys.path.insert(0, refdir)
        import patches.tp_dit as ref_tp_dit
        from h3tp import tp_dit as b200, swiglu_quant
        # The fused FC2 route checks for an sm_100 device before it runs; on these CPU
        # ranks the same contract minus the device check lets the route (and its MAX
        # all-reduce) run on the stand-in kernels.
        def cpu_supported(x, weight, weight_scale, world_size, groupsize):
            try:
                _, kl = swiglu_quant.input_kind(x, weight.shape[1])
            except ValueError:
                return False
            return (kl % 256 == 0 and kl == weight.shape[1] and groupsize == 256
                    and world_size in (1, 2, 4, 8))
        swiglu_quant.supported = cpu_supported
        ref_tp_dit.ColumnParallelLinearINT8 = b200.ColumnParallelLinearINT8
        ref_tp_dit.RowParallelLinearINT8 = b200.RowParallelLinearINT8
        H, heads, hd, F, T, S = 512, 4, 128, 1024, 8, 48
        blk = ref_tp_dit.TPDiTBlockINT8(hidden=H, heads=heads, head_dim=hd, ffn=F, t_dim=T,
                                        rank=rank, world_size=world, device="cpu")
        for name in ("qkv_proj", "out_proj", "fc1", "fc2"):
            assert type(getattr(blk, name)).__module__ == "h3tp.tp_dit", name
        blk.load_from_full_block(_full_block(H, heads, hd, F, T))
        g = torch.Generator().manual_seed(11)
        x = torch.randn((S, H), generator=g)
        t_emb = torch.randn((3, T), generator=g)
        segments = [(0, 20, 0), (20, 33, 2), (33, S, 1)]
        with torch.no_grad():
            out = blk(x.clone(), t_emb, segments)
        assert out.shape == (S, H) and out.dtype == torch.float32
        np.save(os.path.join(outdir, f"r{rank}.npy"), out.numpy())
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        Path(outdir, f"err{rank}.txt").write_text(traceback.format_exc())
        raise
