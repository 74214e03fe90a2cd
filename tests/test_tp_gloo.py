"""Multi-rank host logic on CPU ranks (gloo, world size 2 and 4): the FC2 row chain's
MAX all-reduce, the row-block reduce-scatter / all-gather exchange (uneven row blocks
included), the O-projection route through RowParallelLinearINT8, the INT32 SUM route,
the pre-collective geometry guard and a rank that leaves mid-job.  Kernels are replaced
by the oracle-backed stand-in (tests/oracle_ops.py); the values are compared bit for
bit with the oracle's single-process composition of the reference arithmetic."""
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import tp_worker


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, tmp_path, *args):
    mp.spawn(fn, args=(world, _port(), str(tmp_path), *args), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("mode", ["fused_stored", "fused_recompute"])
def test_fc2_rowblock_exchange_matches_oracle(oracle, tmp_path, world, mode):
    _run(tp_worker.fc2_case, world, tmp_path, mode, "rowblock", True)
    xs, wr, ws, X, G, labels = tp_worker.problem(world)
    ref = X.copy()
    oracle.fc2_fused_stored(xs, wr, ws, out="residual", residual=ref, gate=G, labels=labels)
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npy")
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), f"rank {r}"


def test_fc2_allreduce_transport_tp2(oracle, tmp_path):
    """At TP2 the all-reduce form (the reference's NCCL fp16 SUM) gives the same bits."""
    _run(tp_worker.fc2_case, 2, tmp_path, "fused_stored", "allreduce", True)
    xs, wr, ws, X, G, labels = tp_worker.problem(2)
    ref = X.copy()
    oracle.fc2_fused_stored(xs, wr, ws, out="residual", residual=ref, gate=G, labels=labels)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"r{r}.npy").view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("world,transport", [(2, "allreduce"), (2, "rowblock"), (4, "rowblock")])
def test_fc2_packed_int8_payload(oracle, tmp_path, world, transport):
    """The 'int8_gather' payload: GEMM + group-128 pack per rank, exchange, rank-order
    reconstruction, FP32 dequant and gated residual."""
    _run(tp_worker.fc2_case, world, tmp_path, "fused_recompute", transport, True, "int8_gather")
    xs, wr, ws, X, G, labels = tp_worker.problem(world, N=256)
    rots = [oracle.fc2_rotate(x) for x in xs]
    gmax = np.max(np.stack([m for _, m in rots]), 0)
    qs = [oracle.row_quantize(R, gmax) for R, _ in rots]
    packed = np.stack([oracle.pack8(oracle.int8_gemm(q, w)) for (q, _), w in zip(qs, wr)])
    restored = oracle.unpack8_restore(packed, 256)
    ref = X.copy()
    oracle.dequantize_i32(restored, qs[0][1], ws, out="residual", residual=ref, gate=G, labels=labels)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"r{r}.npy").view(np.uint16), ref.view(np.uint16))


def test_fc2_int32_sum_route(oracle, tmp_path):
    """scaled_transport=False: exact INT32 SUM, then ((acc*a)*w), then the gated add."""
    _run(tp_worker.fc2_case, 2, tmp_path, "fused_recompute", "rowblock", False)
    xs, wr, ws, X, G, labels = tp_worker.problem(2)
    rots = [oracle.fc2_rotate(x) for x in xs]
    gmax = np.maximum(rots[0][1], rots[1][1])
    qs = [oracle.row_quantize(R, gmax) for R, _ in rots]
    total = oracle.int8_gemm(qs[0][0], wr[0]) + oracle.int8_gemm(qs[1][0], wr[1])
    y = oracle.dequantize_i32(total, qs[0][1], ws, out="f32")
    ref = X.copy()
    oracle.gated_add(y, ref, G, labels)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"r{r}.npy").view(np.uint16), ref.view(np.uint16))


def test_o_projection_module_tp2(oracle, tmp_path):
    _run(tp_worker.oproj_case, 2, tmp_path)
    rng = np.random.default_rng(9)
    M, K, N = 29, 512, 64
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (rng.uniform(1e-3, 1e-2, (N, 1)) / 512).astype(np.float32)
    kl = K // 2
    rots = [oracle.fc2_rotate(x[:, r * kl:(r + 1) * kl].copy(), "act_f16") for r in range(2)]
    gmax = np.maximum(rots[0][1], rots[1][1])
    qs = [oracle.row_quantize(R, gmax) for R, _ in rots]
    shift = oracle.transport_shift(K)
    enc = np.stack([oracle.fp16_encode(oracle.int8_gemm(q, w[:, r * kl:(r + 1) * kl]), shift)
                    for r, (q, _) in enumerate(qs)])
    ref = oracle.row_reduce_finish(enc, shift, qs[0][1], s.ravel(), out="f32").astype(np.float16)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"r{r}.npy").view(np.uint16), ref.view(np.uint16))


def test_o_projection_module_partial_groups_tp4(oracle, tmp_path):
    """K = 768 over 4 ranks: 192 columns each, so every rank's slice splits a ConvRot
    group (the O projection at TP 8 in miniature).  The rows are gathered, rotated and
    quantised whole; each rank multiplies its own columns' codes."""
    world, K = 4, 768
    _run(tp_worker.oproj_case, world, tmp_path, K)
    rng = np.random.default_rng(9)
    M, N = 29, 64
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (rng.uniform(1e-3, 1e-2, (N, 1)) / 512).astype(np.float32)
    R, m = oracle.fc2_rotate(x, "act_f16")
    q, a = oracle.row_quantize(R, m)
    kl = K // world
    shift = oracle.transport_shift(K)
    enc = np.stack([oracle.fp16_encode(oracle.int8_gemm(np.ascontiguousarray(q[:, r * kl:(r + 1) * kl]),
                                                        np.ascontiguousarray(w[:, r * kl:(r + 1) * kl])),
                                       shift) for r in range(world)])
    ref = oracle.row_reduce_finish(enc, shift, a, s.ravel(), out="f32").astype(np.float16)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"r{r}.npy").view(np.uint16), ref.view(np.uint16))


def test_unsupported_geometry_raises_before_any_collective(tmp_path):
    _run(tp_worker.guard_case, 2, tmp_path)
    for r in range(2):
        assert (tmp_path / f"r{r}.txt").read_text().startswith("ValueError")


def test_rank_leaving_ends_peer_collective_with_error(tmp_path):
    import time
    ctx = mp.spawn(tp_worker.dead_rank_case, args=(2, _port(), str(tmp_path)), nprocs=2, join=False)
    t0 = time.time()
    while not ctx.join(timeout=5):
        assert time.time() - t0 < 120, "surviving rank did not finish"
    assert (tmp_path / "r1.txt").read_text() == "left"
    msg = (tmp_path / "r0.txt").read_text()
    assert msg.startswith("error after"), msg
