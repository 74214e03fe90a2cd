"""Host-side API contracts that need no GPU: operator policy values and validation,
module constructors and parameter layouts (tp_dit.py:25-162), dispatch guards, and the
absence of any CPU fallback in the kernel wrappers."""
import dataclasses

import pytest
import torch


def test_policy_defaults_and_validation():
    from h3tp.h3_operator_policy import H3OperatorPolicy
    p = H3OperatorPolicy()
    assert p.row_linear_backend == "b200_scaled_fp16" and p.scaled_transport
    # the reference's defaults (patches/h3_operator_policy.py:14): fused_stored, and FC1
    # returning fp16 [gate|up] unless the FP32 SwiGLU epilogue is asked for
    assert p.fc2_quantizer == "fused_stored" and not p.fc1_swiglu_epilogue
    assert p.column_linear_backend == "b200"
    # the reference's own values stay accepted (h3_operator_policy.py:9-41)
    ref = H3OperatorPolicy(row_linear_backend="tilelang_scaled_fp16", fc2_quantizer="fused_stored",
                           column_linear_backend="cuda_int8_tilelang")
    assert ref.scaled_transport
    assert not H3OperatorPolicy(row_linear_backend="native").scaled_transport
    for bad in (dict(row_linear_backend="x"), dict(fc2_quantizer="x"), dict(column_linear_backend="x"),
                dict(row_transport="ring"), dict(quant_division="approx"), dict(dit_fused_row_gate=1),
                dict(row_payload="int4"), dict(fc2_max_exchange="ring")):
        with pytest.raises(ValueError):
            H3OperatorPolicy(**bad)
    with pytest.raises(dataclasses.FrozenInstanceError):
        p.fc2_quantizer = "native"


def test_policy_max_exchange_default():
    from h3tp.h3_operator_policy import H3OperatorPolicy
    p = H3OperatorPolicy()
    assert p.row_transport == "p2p" and p.fc2_max_exchange == "peer"
    assert H3OperatorPolicy(fc2_max_exchange="nccl").fc2_max_exchange == "nccl"


def test_peer_epochs_skip_zero():
    from h3tp import peer
    assert peer.next_epoch(0) == 1 and peer.next_epoch(1) == 2
    assert peer.next_epoch(0xFFFFFFFE) == 0xFFFFFFFF
    assert peer.next_epoch(0xFFFFFFFF) == 1  # wraps past the zeroed flags' tag


@pytest.mark.parametrize("width,rows", [(3072, 32768), (512, 1), (264, 77), (13824, 4099)])
def test_peer_workspace_layout(width, rows):
    """Flags, partial, final rows and row-maximum slots of the peer workspace: disjoint,
    256-byte aligned, and large enough for the fp16 partial, the packed INT8 rows
    (width / 128 groups of 132 bytes) and 8 slots of 8 bytes per row."""
    from h3tp import peer
    lay = peer.layout(width, rows)
    areas = [(0, peer.FLAGS_BYTES), (lay["partial_off"], lay["final_off"]),
             (lay["final_off"], lay["slots_off"]), (lay["slots_off"], lay["nbytes"])]
    for (a0, a1), (b0, _) in zip(areas, areas[1:]):
        assert a1 <= b0
    for off in (lay["partial_off"], lay["final_off"], lay["slots_off"]):
        assert off % 256 == 0
    assert lay["final_off"] - lay["partial_off"] >= rows * width * 2
    assert lay["final_off"] - lay["partial_off"] >= rows * (width // 128) * 132
    assert lay["slots_off"] - lay["final_off"] >= rows * width * 2
    assert lay["nbytes"] - lay["slots_off"] >= rows * 8 * 8


def test_tensor_flow_policy():
    from h3tp.h3_tensor_flow import TensorFlowPolicy
    assert TensorFlowPolicy().divisor == 512.0
    with pytest.raises(ValueError):
        TensorFlowPolicy(residual_exponent=13)
    with pytest.raises(ValueError):
        TensorFlowPolicy(mode="fp8")


def test_module_parameter_layouts():
    from h3tp.tp_dit import ColumnParallelLinearINT8, RowParallelLinearINT8
    c = ColumnParallelLinearINT8(512, 3 * 1024, rank=1, world_size=4, components=3, device="cpu")
    assert c.weight.shape == (768, 512) and c.weight.dtype == torch.int8
    assert c.weight_scale.shape == (768, 1) and c.weight_scale.dtype == torch.float32
    assert not c.weight.requires_grad
    r = RowParallelLinearINT8(8192, 3072, rank=3, world_size=8, device="cpu")
    assert r.weight.shape == (3072, 1024) and r.weight_scale.shape == (3072, 1)
    full = torch.arange(3072 * 8192, dtype=torch.int64).remainder(251).sub(125).to(torch.int8).reshape(3072, 8192)
    r.load_shard_from_full(full, torch.ones(3072, 1))
    assert torch.equal(r.weight, full[:, 3 * 1024:4 * 1024])
    with pytest.raises(AssertionError):
        RowParallelLinearINT8(1000, 64, world_size=3, device="cpu")


def test_row_parallel_requires_reduction_and_group():
    from h3tp.tp_dit import RowParallelLinearINT8
    r = RowParallelLinearINT8(512, 64, rank=0, world_size=2, device="cpu")
    with pytest.raises(ValueError):
        r(torch.zeros(3, 256, dtype=torch.float16), reduce_sum=False)
    with pytest.raises(RuntimeError):
        r(torch.zeros(3, 256, dtype=torch.float16))  # no initialised TP group of 2


def test_kernel_wrappers_have_no_cpu_fallback():
    from h3tp import ops
    q = torch.zeros((4, 64), dtype=torch.int8)
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.int8_gemm_i32(q, q)
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.column_quantize(torch.zeros((4, 256), dtype=torch.float16))
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.swiglu_rotate_quantize_local(torch.zeros((4, 512), dtype=torch.float16))


def test_fc2_input_classification():
    from h3tp.swiglu_quant import input_kind, supported
    assert input_kind(torch.zeros(2, 1024, dtype=torch.float16), 512) == ("gateup_f16", 512)
    assert input_kind(torch.zeros(2, 512, dtype=torch.float32), 512) == ("act_f32", 512)
    assert input_kind(torch.zeros(2, 512, dtype=torch.float16), 512) == ("act_f16", 512)
    with pytest.raises(ValueError):
        input_kind(torch.zeros(2, 1024, dtype=torch.float32), 512)
    with pytest.raises(ValueError):
        input_kind(torch.zeros(2, 512, dtype=torch.bfloat16), 512)
    w = torch.zeros(128, 512, dtype=torch.int8)
    assert not supported(torch.zeros(2, 1024, dtype=torch.float16), w, torch.ones(128), 2, 256)  # CPU


def test_row_blocks_cover_rows_once():
    from h3tp.comm import row_blocks
    for rows in (0, 1, 7, 37, 32768):
        for world in (1, 2, 3, 4, 8):
            blocks = row_blocks(rows, world)
            assert len(blocks) == world
            cover = [i for a, b in blocks for i in range(a, b)]
            assert cover == list(range(rows))


def test_transport_shift_generalisation():
    from h3tp import ops, transport
    assert transport.shift_for(7168) == 12 and transport.shift_for(3584) == 11
    assert transport.shift_for(8192 // 8, 8) == transport.shift_for(8192 // 2, 2) == 12
    assert ops.transport_shift(3072) == 10


class _FakeComm:
    """Duck-typed torch.distributed of world 2 that records collective calls."""
    def __init__(self):
        self.calls = []

    def is_initialized(self):
        return True

    def get_world_size(self):
        return 2

    def get_rank(self):
        return 0

    def all_reduce(self, t, op=None):
        self.calls.append("all_reduce")


class _FakeWorkspace:
    def __init__(self):
        self.seen = []

    def quantize_rows(self, x, kind, division):
        self.seen.append((tuple(x.shape), kind, division))
        rows, width = x.shape[0], (x.shape[1] // 2 if kind == "gateup_f16" else x.shape[1])
        return (torch.zeros((rows, width), dtype=torch.int8),
                torch.ones((rows, 1), dtype=torch.float32))


@pytest.mark.parametrize("dtype,width,kind", [(torch.float16, 1024, "gateup_f16"),
                                              (torch.float32, 512, "act_f32")])
def test_prepare_with_peer_workspace_takes_one_pass(dtype, width, kind):
    """At TP > 1 with a peer workspace, prepare() hands the whole activation to the
    workspace's single-pass producer and issues no NCCL MAX; consume_input releases the
    caller's storage afterwards (tilelang_swiglu_quant.py:81-85)."""
    from h3tp import swiglu_quant
    comm, ws = _FakeComm(), _FakeWorkspace()
    x = torch.zeros((3, 5, width), dtype=dtype)
    q, s = swiglu_quant.prepare(x, comm, "fused_recompute", consume_input=True, division="rn",
                                local_k=512, peer_workspace=ws)
    assert ws.seen == [((15, width), kind, "rn")]
    assert comm.calls == []
    assert q.shape == (15, 512) and s.shape == (15, 1)
    assert x.numel() == 0  # storage released


def test_prepare_rejects_partial_groups_before_the_workspace():
    from h3tp import swiglu_quant
    comm, ws = _FakeComm(), _FakeWorkspace()
    with pytest.raises(ValueError):
        swiglu_quant.prepare(torch.zeros((4, 2 * 384), dtype=torch.float16), comm,
                             peer_workspace=ws)
    assert ws.seen == [] and comm.calls == []


@pytest.mark.parametrize("rows,chunks", [(32768, 4), (2085, 3), (4096, 2), (300, 4), (256, 8),
                                         (1, 2), (32768 + 77, 4)])
def test_pipeline_bounds_tile_the_rows(rows, chunks):
    """The pipelined MLP forward's row chunks cover every row once, start on whole
    256-row tiles and are never empty."""
    from h3tp.tp_dit import pipeline_bounds
    b = pipeline_bounds(rows, chunks)
    assert b[0][0] == 0 and b[-1][1] == rows
    assert all(x[1] == y[0] for x, y in zip(b, b[1:]))
    assert all(a < e for a, e in b) and all(a % 256 == 0 for a, _ in b)
    assert len(b) <= max(1, chunks)


def test_policy_pipeline_chunks_validation():
    from h3tp.h3_operator_policy import H3OperatorPolicy
    assert H3OperatorPolicy().mlp_pipeline_chunks == 1
    for bad in (-1, 65, 2.0, True):
        with pytest.raises(ValueError):
            H3OperatorPolicy(mlp_pipeline_chunks=bad)


def test_p2p_exchange_form_override(monkeypatch):
    """The p2p exchange form: the measured default per TP size, overridden by
    H3_P2P_EXCHANGE (read at import); either form gives the same bits."""
    import importlib
    from h3tp import peer
    for env, want in (("push", True), ("pull", False), ("dma", False)):
        monkeypatch.setenv("H3_P2P_EXCHANGE", env)
        importlib.reload(peer)
        assert all(peer.pushes(w) is want for w in (2, 4, 8))
        assert all(peer.exchange_form(w) == env for w in (2, 4, 8))
    monkeypatch.delenv("H3_P2P_EXCHANGE", raising=False)
    importlib.reload(peer)
    assert all(isinstance(peer.pushes(w), bool) for w in (2, 4, 8))


def test_bench_reference_arm_json_contract():
    """bench.py --impl reference on a tiny block: one JSON line with the contract's keys,
    the e2e object of a host-only run and the CPU baseline it describes."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference",
                        "--tokens", "512", "--hidden", "256", "--ffn", "512", "--steps", "2",
                        "--warmup", "1", "--ref-rows", "64"],
                       capture_output=True, text=True, timeout=300, cwd=str(root))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"] == "dit_mlp_block" and d["config"]["M"] == 512
