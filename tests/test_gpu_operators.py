"""Operator-level parity on the GPU: the reference-facing modules and functions
(tp_dit, dit_column_linear, swiglu_quant, row_quant, transport, dit_fusion) against
the CPU oracle's composition of the reference arithmetic.

Multi-rank arithmetic is emulated on one GPU by running each rank's kernels on its
own shard and combining them the way the collectives do (elementwise MAX of the row
maxima; the rank-ordered partial reduction of h3_row_reduce_finish).  The NCCL
plumbing itself is covered by tests/test_gpu_tp_nccl.py on >= 2 GPUs and by the gloo
tests on the CPU.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


def _eq(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    v = {1: np.uint8, 2: np.uint16, 4: np.uint32}[a.itemsize]
    bad = np.flatnonzero(a.view(v) != b.view(v))
    assert bad.size == 0, f"{bad.size}/{a.size} differ, first {a.flat[bad[0]]} vs {b.flat[bad[0]]}"


def _weights(rng, n, k, fold=1.0):
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = (rng.uniform(1e-3, 1e-2, size=(n, 1)) / fold).astype(np.float32)
    return w, s


def test_column_parallel_module_qkv(cuda_device, oracle):
    from h3tp.tp_dit import ColumnParallelLinearINT8
    rng = np.random.default_rng(1)
    M, hidden, world = 77, 512, 2
    x = rng.standard_normal((M, hidden)).astype(np.float16)
    w, s = _weights(rng, 3 * 256 * 2, hidden)
    for rank in range(world):
        mod = ColumnParallelLinearINT8(hidden, w.shape[0], rank, world, components=3, device=cuda_device)
        mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(s))
        wr, sr = oracle.packed_rows(w, s, rank, world, 3)
        _eq(_np(mod.weight), wr)
        with torch.no_grad():
            y = mod(_t(x, cuda_device))
        ref, _ = oracle.column_linear(x, wr, sr.ravel(), convrot=True)
        _eq(_np(y), ref)


def test_column_linear_no_rotation_with_bias(cuda_device, oracle):
    """BASELINE config 1 form: no rotation, per-row absmax quant, INT32, FP32 dequant."""
    from h3tp.dit_column_linear import column_linear
    rng = np.random.default_rng(2)
    x = rng.standard_normal((64, 3072)).astype(np.float32)
    x[:, rng.permutation(3072)[:30]] *= 20
    x = x.astype(np.float16)
    w, s = _weights(rng, 384, 3072)
    b = (rng.standard_normal(384) * 0.02).astype(np.float32)
    y = column_linear(_t(x, cuda_device), _t(w, cuda_device), _t(s, cuda_device), convrot=False,
                      bias=_t(b, cuda_device))
    q, a = oracle.column_quantize(x, False)
    _eq(_np(y), oracle.column_epilogue(oracle.int8_gemm(q, w), a, s.ravel(), b))


def _baseline_config1(seed=0):
    """BASELINE config 1 exactly: X fp16 [1024, 3072] ~ N(0, 1) with 1% of the columns
    (a seeded randperm, 30 columns) scaled x20; W int8 [3072, 3072] uniform in
    [-127, 127]; per-output-channel fp32 scales uniform in [1e-3, 1e-2]; bias
    ~ N(0, 0.02); seed 0."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((1024, 3072), generator=g)
    cols = torch.randperm(3072, generator=g)[:30]
    x[:, cols] *= 20.0
    w = torch.randint(-127, 128, (3072, 3072), generator=g, dtype=torch.int8)
    s = (torch.rand((3072, 1), generator=g) * 9e-3 + 1e-3).float()
    b = (torch.randn(3072, generator=g) * 0.02).float()
    return x.half().numpy(), w.numpy(), s.numpy(), b.numpy()


@pytest.mark.parametrize("bias", [False, True])
def test_baseline_config1_column_linear(cuda_device, oracle, bias):
    """The single W8A8 linear of BASELINE config 1 (M = 1024, K = N = 3072, no
    rotation, dynamic per-row quant, INT32 accumulate, FP32 dequant, fp16 out) through
    the public column_linear: codes, row scales, INT32 accumulators and the fp16 output
    all bit-exact against the oracle."""
    from h3tp import ops
    from h3tp.dit_column_linear import column_linear
    x, w, s, b = _baseline_config1()
    b = b if bias else None
    xd, wd, sd = _t(x, cuda_device), _t(w, cuda_device), _t(s, cuda_device)
    q_ref, a_ref = oracle.column_quantize(x, False)
    q, a = ops.column_quantize(xd, False)
    _eq(_np(q), q_ref)
    _eq(_np(a).ravel(), a_ref.ravel())
    acc_ref = oracle.int8_gemm(q_ref, w)
    _eq(_np(ops.int8_gemm_i32(q, wd)), acc_ref)
    y = column_linear(xd, wd, sd, convrot=False, bias=None if b is None else _t(b, cuda_device))
    _eq(_np(y), oracle.column_epilogue(acc_ref, a_ref, s.ravel(), b))


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("mode", ["fused_stored", "fused_recompute"])
def test_fc2_chain_emulated_tp(cuda_device, oracle, world, mode):
    """FC2 fused_stored chain at TP=world, one GPU: codes, INT32 partials and the
    fp32 output are bit-exact against the oracle."""
    from h3tp import ops, transport
    rng = np.random.default_rng(world * 3 + len(mode))
    M, K, N = 70, 1024 * world, 384
    gate = rng.standard_normal((M, K)).astype(np.float32)
    gate[::9] *= rng.standard_t(3, size=(len(gate[::9]), K)).astype(np.float32)
    up = rng.standard_normal((M, K)).astype(np.float32)
    w, s = _weights(rng, N, K, fold=512)
    kl = K // world
    xs = [np.concatenate([gate[:, r * kl:(r + 1) * kl], up[:, r * kl:(r + 1) * kl]], 1).astype(np.float16)
          for r in range(world)]
    ws = [w[:, r * kl:(r + 1) * kl].copy() for r in range(world)]
    ref, qs_ref, parts_ref = oracle.fc2_fused_stored(xs, ws, s.ravel(), out="f32")
    xd = [_t(x, cuda_device) for x in xs]
    if world == 1:
        from h3tp.swiglu_quant import row_linear
        y = row_linear(xd[0], _t(ws[0], cuda_device), _t(s, cuda_device), None, mode=mode)
        _eq(_np(y), ref)
        return
    maxes = [ops.swiglu_rotate_max(x, "gateup_f16", store=(mode == "fused_stored")) for x in xd]
    gmax = torch.stack([m for _, m in maxes]).amax(0)
    shift = transport.shift_for(kl, world)
    payload = []
    for r in range(world):
        if mode == "fused_stored":
            q, sc = ops.row_quantize(maxes[r][0], gmax)
        else:
            q, sc = ops.swiglu_rotate_quantize(xd[r], gmax, "gateup_f16")
        _eq(_np(q), qs_ref[r][0])
        _eq(_np(sc).ravel(), qs_ref[r][1])
        _eq(_np(ops.int8_gemm_i32(q, _t(ws[r], cuda_device))), parts_ref[r])
        payload.append(ops.int8_gemm_row_encode(q, _t(ws[r], cuda_device), shift))
    y = ops.row_reduce_finish(torch.stack(payload), shift, sc, _t(s, cuda_device))
    _eq(_np(y), ref)


def test_row_parallel_module_tp1_residual_gate(cuda_device, oracle):
    """RowParallelLinearINT8(input_act='swiglu', residual, gate, segments) at TP=1."""
    from h3tp.h3_operator_policy import H3OperatorPolicy
    from h3tp.tp_dit import RowParallelLinearINT8
    rng = np.random.default_rng(4)
    M, kl, N = 96, 2048, 512
    x = rng.standard_normal((M, 2 * kl)).astype(np.float16)
    w, s = _weights(rng, N, kl, fold=512)
    X = rng.standard_normal((M, N)).astype(np.float16)
    gate = rng.standard_normal((3, N)).astype(np.float32)
    segments = [(0, 40, 0), (40, 70, 2), (70, 96, 1)]
    labels = np.zeros(M, np.int32)
    for a, b, r in segments:
        labels[a:b] = r
    mod = RowParallelLinearINT8(kl, N, 0, 1, device=cuda_device)
    mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(s))
    mod.operator_policy = H3OperatorPolicy()
    Xd = _t(X, cuda_device)
    with torch.no_grad():
        out = mod(_t(x, cuda_device), input_act="swiglu", residual=Xd, gate=_t(gate, cuda_device),
                  segments=segments)
    assert out.data_ptr() == Xd.data_ptr()
    ref = X.copy()
    oracle.fc2_fused_stored([x], [w], s.ravel(), out="residual", residual=ref, gate=gate, labels=labels)
    _eq(_np(Xd), ref)


def test_mlp_block_tp1_matches_oracle(cuda_device, oracle):
    """TPDiTMLPINT8 (FC1 SwiGLU epilogue -> FC2 fused chain -> residual add), TP=1."""
    from h3tp.tp_dit import TPDiTMLPINT8
    rng = np.random.default_rng(5)
    M, hidden, ffn = 130, 768, 1536
    h = rng.standard_normal((M, hidden)).astype(np.float16)
    X = rng.standard_normal((M, hidden)).astype(np.float16)
    w1, s1 = _weights(rng, 2 * ffn, hidden)
    w2, s2 = _weights(rng, hidden, ffn, fold=512)
    mlp = TPDiTMLPINT8(hidden, ffn, 0, 1, device=cuda_device)
    mlp.fc1.load_shard_from_full(torch.from_numpy(w1), torch.from_numpy(s1))
    mlp.fc2.load_shard_from_full(torch.from_numpy(w2), torch.from_numpy(s2))
    Xd = _t(X, cuda_device)
    with torch.no_grad():
        mlp(Xd, _t(h, cuda_device))
    q, a = oracle.column_quantize(h, True)
    act = oracle.swiglu_epilogue(oracle.int8_gemm(q, w1), a, s1.ravel())
    ref = X.copy()
    oracle.fc2_fused_stored([act], [w2], s2.ravel(), out="residual", residual=ref, kind="act_f32")
    _eq(_np(Xd), ref)


def test_fc1_swiglu_epilogue_equals_fp16_gateup_route(cuda_device):
    """The FP32 SwiGLU FC1 epilogue and the reference's fp16 [gate|up] store followed
    by the FC2 producer's SwiGLU give identical INT8 codes (same values, same bytes)."""
    from h3tp import ops
    from h3tp.dit_column_linear import column_linear
    rng = np.random.default_rng(6)
    h = _t(rng.standard_normal((200, 1024)).astype(np.float16), cuda_device)
    w, s = _weights(rng, 2 * 512, 1024)
    wd, sd = _t(w, cuda_device), _t(s, cuda_device)
    gateup = column_linear(h, wd, sd)
    act = column_linear(h, wd, sd, swiglu=True)
    q1, s1, m1 = ops.swiglu_rotate_quantize_local(gateup, "gateup_f16")
    q2, s2, m2 = ops.swiglu_rotate_quantize_local(act, "act_f32")
    assert torch.equal(q1, q2) and torch.equal(s1, s2) and torch.equal(m1, m2)


def test_o_projection_row_emulated_tp2(cuda_device, oracle):
    """O projection: local ConvRot of owned groups, global max, GEMM, fp16 transport."""
    from h3tp import ops, transport
    rng = np.random.default_rng(8)
    M, K, N, world = 50, 1024, 256, 2
    xs_full = rng.standard_normal((M, K)).astype(np.float16)
    w, s = _weights(rng, N, K, fold=512)
    kl = K // world
    maxes, qs, payload = [], [], []
    for r in range(world):
        xr = _t(xs_full[:, r * kl:(r + 1) * kl], cuda_device)
        maxes.append(ops.swiglu_rotate_max(xr, "act_f16", store=False)[1])
    gmax = torch.stack(maxes).amax(0)
    shift = transport.shift_for(kl, world)
    R = [oracle.fc2_rotate(xs_full[:, r * kl:(r + 1) * kl], "act_f16") for r in range(world)]
    gref = np.maximum(R[0][1], R[1][1])
    for r in range(world):
        xr = _t(xs_full[:, r * kl:(r + 1) * kl], cuda_device)
        q, sc = ops.swiglu_rotate_quantize(xr, gmax, "act_f16")
        qr, sr = oracle.row_quantize(R[r][0], gref)
        _eq(_np(q), qr)
        payload.append(ops.int8_gemm_row_encode(q, _t(w[:, r * kl:(r + 1) * kl].copy(), cuda_device), shift))
    y = ops.row_reduce_finish(torch.stack(payload), shift, sc, _t(s, cuda_device))
    parts = np.stack([oracle.fp16_encode(oracle.int8_gemm(oracle.row_quantize(R[r][0], gref)[0],
                                                          w[:, r * kl:(r + 1) * kl]), shift)
                      for r in range(world)])
    _eq(_np(y), oracle.row_reduce_finish(parts, shift, sr, s.ravel()))


def test_te_shared_column_linears_k5120(cuda_device, oracle):
    """TE (Qwen3-VL) column shapes: one rotation + quantisation of a K = 5120 input
    shared by two projections (dit_column_linear.py:70-96)."""
    from h3tp.dit_column_linear import shared_column_linears
    rng = np.random.default_rng(12)
    x = rng.standard_normal((96, 5120)).astype(np.float32)
    x[:, rng.permutation(5120)[:51]] *= 20
    x = x.astype(np.float16)
    projections = [_weights(rng, 1536, 5120), _weights(rng, 512, 5120)]
    with torch.no_grad():
        outs = shared_column_linears(_t(x, cuda_device),
                                     [(_t(w, cuda_device), _t(s, cuda_device)) for w, s in projections])
    for (w, s), y in zip(projections, outs):
        ref, _ = oracle.column_linear(x, w, s.ravel(), convrot=True)
        _eq(_np(y), ref)


def test_te_row_linear_parts_k12800(cuda_device, oracle):
    """TE row shape: separate gate / up inputs of K = 12800 through row_linear_parts
    (h3_operator_policy.py:240-255), the fused FC2 route at TP = 1."""
    from h3tp.h3_operator_policy import H3OperatorPolicy, row_linear_parts
    from h3tp.tp_dit import RowParallelLinearINT8
    rng = np.random.default_rng(13)
    M, kl, N = 64, 12800, 512
    gate = rng.standard_normal((M, kl)).astype(np.float16)
    up = rng.standard_normal((M, kl)).astype(np.float16)
    w, s = _weights(rng, N, kl, fold=512)
    mod = RowParallelLinearINT8(kl, N, 0, 1, device=cuda_device)
    mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(s))
    mod.operator_policy = H3OperatorPolicy()

    def fallback(*args):
        raise AssertionError("the fused route must apply")

    with torch.no_grad():
        y = row_linear_parts(mod, _t(gate, cuda_device), _t(up, cuda_device), fallback, None)
    ref, _, _ = oracle.fc2_fused_stored([np.concatenate([gate, up], 1)], [w], s.ravel(), out="f32")
    _eq(_np(y), ref)


def test_fused_norm_then_column_parallel_qkv(cuda_device, oracle):
    """dit_fusion.modulated_norm_quantize feeding ColumnParallelLinearINT8.forward_quantized
    gives the bits of the unfused route (norm -> fp16 h -> column linear)."""
    from types import SimpleNamespace
    from h3tp.dit_fusion import modulated_norm, modulated_norm_quantize
    from h3tp.tp_dit import ColumnParallelLinearINT8
    rng = np.random.default_rng(14)
    M, hidden = 50, 1024
    x = (rng.standard_normal((M, hidden)) * 2).astype(np.float16)
    norm = SimpleNamespace(normalized_shape=(hidden,), eps=1e-6,
                           weight=_t(rng.uniform(.5, 1.5, hidden).astype(np.float32), cuda_device))
    shift = (rng.standard_normal((3, hidden)) * .1).astype(np.float32)
    scale = (rng.standard_normal((3, hidden)) * .1).astype(np.float32)
    segments = [(0, 20, 0), (20, 50, 2)]
    w, s = _weights(rng, 3 * 256, hidden)
    mod = ColumnParallelLinearINT8(hidden, w.shape[0], 0, 1, components=3, device=cuda_device)
    mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(s))
    xd, sh, sc = _t(x, cuda_device), _t(shift, cuda_device), _t(scale, cuda_device)
    with torch.no_grad():
        q, a = modulated_norm_quantize(norm, xd, sh, sc, segments)
        y = mod.forward_quantized(q, a)
        h = modulated_norm(norm, xd, sh, sc, segments)
        y_unfused = mod(h)
    labels = np.concatenate([np.zeros(20, np.int32), np.full(30, 2, np.int32)])
    h_ref = oracle.modulated_norm(x, _np(norm.weight), 1e-6, shift, scale, labels)
    _eq(_np(h), h_ref)
    ref, _ = oracle.column_linear(h_ref, w, s.ravel(), convrot=True)
    _eq(_np(y), ref)
    _eq(_np(y_unfused), ref)


def test_unsupported_geometry_raises_before_launch(cuda_device):
    from h3tp import ops
    x = torch.zeros((4, 300), dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError):
        ops.swiglu_rotate_max(x, "act_f16")      # width not a multiple of 256
    q = torch.zeros((4, 40), dtype=torch.int8, device=cuda_device)
    w = torch.zeros((8, 40), dtype=torch.int8, device=cuda_device)
    with pytest.raises(ValueError):
        ops.int8_gemm_i32(q, w)                  # K not a multiple of 16
    with pytest.raises(ValueError):
        ops.int8_gemm_i32(q.cpu(), w.cpu())      # no CPU fallback


def _linear_block_weights(rng, hidden, ffn):
    wqkv, sqkv = _weights(rng, 3 * hidden, hidden)
    wo, so = _weights(rng, hidden, hidden, fold=512)
    w1, s1 = _weights(rng, 2 * ffn, hidden)
    w2, s2 = _weights(rng, hidden, ffn, fold=512)
    return wqkv, sqkv, wo, so, w1, s1, w2, s2


def test_linear_block_tp1_matches_oracle(cuda_device, oracle):
    """TPDiTLinearBlockINT8 (QKV -> O + gated residual -> FC1 -> FC2 + gated residual,
    BASELINE config 4's linear set) at TP 1, bit-exact against oracle.linear_block."""
    from h3tp.tp_dit import TPDiTLinearBlockINT8
    rng = np.random.default_rng(31)
    M, hidden, ffn = 300, 512, 1024
    W = _linear_block_weights(rng, hidden, ffn)
    X = rng.standard_normal((M, hidden)).astype(np.float16)
    G1 = rng.standard_normal((3, hidden)).astype(np.float32)
    G2 = rng.standard_normal((3, hidden)).astype(np.float32)
    segments = [(0, 100, 2), (100, 300, 0)]
    labels = np.array([2] * 100 + [0] * 200, np.int32)
    blk = TPDiTLinearBlockINT8(hidden, ffn, 0, 1, device=cuda_device)
    for mod, (w, sc) in zip((blk.qkv_proj, blk.out_proj, blk.fc1, blk.fc2),
                            zip(W[0::2], W[1::2])):
        mod.load_shard_from_full(torch.from_numpy(w), torch.from_numpy(sc))
    x = _t(X, cuda_device)
    with torch.no_grad():
        y = blk(x, gate_msa=_t(G1, cuda_device), gate_mlp=_t(G2, cuda_device), segments=segments)
    ref = oracle.linear_block(X, *W, 1, G1, G2, labels)
    _eq(_np(y), ref)
