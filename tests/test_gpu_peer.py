"""The peer-memory row transport kernels (h3_peer_reduce, h3_peer_gather) on one GPU.

Each emulated rank gets its own workspace buffer on the same device, and its row GEMM
(h3_int8_gemm_row_encode) writes the encoded partial into that buffer; the partials
are checked against the oracle's INT8 GEMM + encode.  Every flag a reduce or
gather kernel waits for is set before that kernel is launched (by an earlier kernel
of the same stream or by the test), so no kernel ever waits for another one that runs
at the same time.  The reduced, gated residual of every rank is compared bit for bit
with the oracle's rank-order reduction; a flag that nothing sets checks the bounded
wait.  The same kernels across real NCCL ranks are covered by
tests/test_gpu_tp_nccl.py."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FLAGS, READY, DONE = 1024, 0, 256


def _region(rows, width):
    return -(-rows * width * 2 // 256) * 256


def _buffers(dev, world, rows, width):
    partial = FLAGS
    final = FLAGS + _region(rows, width)
    nbytes = final + _region(rows, width)
    return [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(world)], partial, final


def _set(buf, region, ranks, epoch):
    flags = buf[:FLAGS].view(torch.int32)
    for w in ranks:
        flags[region // 4 + w] = epoch


@pytest.mark.parametrize("world,rows,width,k", [(2, 130, 512, 512), (4, 77, 264, 256),
                                                (8, 99, 1024, 256)])
def test_peer_transport_bit_exact(cuda_device, oracle, world, rows, width, k):
    from h3tp import _native, ops, transport
    rng = np.random.default_rng(world)
    shift = transport.shift_for(k, world)
    qs = [rng.integers(-128, 128, size=(rows, k), dtype=np.int8) for _ in range(world)]
    ws = [rng.integers(-127, 128, size=(width, k), dtype=np.int8) for _ in range(world)]
    enc = np.stack([oracle.fp16_encode(oracle.int8_gemm(q, w), shift) for q, w in zip(qs, ws)])
    a = rng.uniform(1e-4, 1e-2, size=rows).astype(np.float32)
    s = rng.uniform(1e-5, 1e-4, size=width).astype(np.float32)
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((3, width)).astype(np.float32)
    labels = rng.integers(0, 3, size=rows).astype(np.int32)
    ref = X.copy()
    oracle.row_reduce_finish(enc, shift, a, s, out="residual", residual=ref, gate=G, labels=labels)

    dev = cuda_device
    bufs, roff, foff = _buffers(dev, world, rows, width)
    bases = [b.data_ptr() for b in bufs]
    A, S = torch.from_numpy(a).to(dev), torch.from_numpy(s).to(dev)
    Gd, L = torch.from_numpy(G).to(dev), torch.from_numpy(labels).to(dev)
    qd = [torch.from_numpy(q).to(dev) for q in qs]
    wd = [torch.from_numpy(w).to(dev) for w in ws]
    res = [torch.from_numpy(X.copy()).to(dev) for _ in range(world)]
    for epoch in (1, 2):  # the second call reuses the buffers and advances the epoch
        for r in range(world):
            res[r].copy_(torch.from_numpy(X))
            part = bufs[r][roff:roff + rows * width * 2].view(torch.float16).view(rows, width)
            ops.int8_gemm_row_encode(qd[r], wd[r], shift, out=part)
        torch.cuda.synchronize()
        for r in range(world):
            got = bufs[r][roff:roff + rows * width * 2].view(torch.float16).cpu().numpy()
            assert np.array_equal(got.view(np.uint16), enc[r].reshape(-1).view(np.uint16)), r
        for b in bufs:
            _set(b, READY, range(world), epoch)
        for r in range(world):
            ops.peer_reduce(bases, world, r, 0, roff, foff, rows, width, shift, A, S, res[r], Gd, L,
                            epoch)
        for r in range(world):
            ops.peer_gather(bases, world, r, 0, foff, rows, width, res[r], epoch)
        torch.cuda.synchronize()
        for r in range(world):
            got = res[r].cpu().numpy()
            assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), f"rank {r} epoch {epoch}"
            flags = bufs[r][:FLAGS].view(torch.int32)
            assert (flags[DONE // 4: DONE // 4 + world].cpu().numpy() == epoch).all()
            assert int(flags[128]) == 0  # counter reset
    assert _native.device_error(dev.index or 0) == 0


@pytest.mark.parametrize("world,rows,width,k", [(2, 130, 512, 512), (4, 77, 264, 256),
                                                (8, 99, 1024, 256), (2, 1030, 3072, 1024)])
def test_peer_transport_pushed_bit_exact(cuda_device, oracle, world, rows, width, k):
    """The fused reduce-scatter: each emulated rank's row GEMM stores every partial row
    into the buffer of the rank that owns it (h3_int8_gemm_row_encode_push, slot row
    rank * per + local row), the owner sums its slots from local memory
    (h3_peer_reduce_pushed); slots and residuals against the oracle, bit for bit."""
    from h3tp import _native, ops, transport
    rng = np.random.default_rng(world + 40)
    shift = transport.shift_for(k, world)
    qs = [rng.integers(-128, 128, size=(rows, k), dtype=np.int8) for _ in range(world)]
    ws = [rng.integers(-127, 128, size=(width, k), dtype=np.int8) for _ in range(world)]
    enc = np.stack([oracle.fp16_encode(oracle.int8_gemm(q, w), shift) for q, w in zip(qs, ws)])
    a = rng.uniform(1e-4, 1e-2, size=rows).astype(np.float32)
    s = rng.uniform(1e-5, 1e-4, size=width).astype(np.float32)
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((3, width)).astype(np.float32)
    labels = rng.integers(0, 3, size=rows).astype(np.int32)
    ref = X.copy()
    oracle.row_reduce_finish(enc, shift, a, s, out="residual", residual=ref, gate=G, labels=labels)

    dev = cuda_device
    per = -(-rows // world)
    bufs, roff, foff = _buffers(dev, world, world * per, width)
    bases = [b.data_ptr() for b in bufs]
    A, S = torch.from_numpy(a).to(dev), torch.from_numpy(s).to(dev)
    Gd, L = torch.from_numpy(G).to(dev), torch.from_numpy(labels).to(dev)
    qd = [torch.from_numpy(q).to(dev) for q in qs]
    wd = [torch.from_numpy(w).to(dev) for w in ws]
    res = [torch.from_numpy(X.copy()).to(dev) for _ in range(world)]
    for epoch in (1, 2):
        for r in range(world):
            res[r].copy_(torch.from_numpy(X))
            ops.int8_gemm_row_encode_push(qd[r], wd[r], shift, bases, world, r, roff)
        torch.cuda.synchronize()
        for o in range(world):
            slots = bufs[o][roff:roff + world * per * width * 2].view(torch.float16)
            slots = slots.view(world, per, width).cpu().numpy()
            lo, hi = o * per, min(rows, (o + 1) * per)
            for r in range(world):
                got = slots[r, :hi - lo].view(np.uint16)
                assert np.array_equal(got, enc[r][lo:hi].view(np.uint16)), (o, r)
        for b in bufs:
            _set(b, READY, range(world), epoch)
        for r in range(world):
            ops.peer_reduce(bases, world, r, 0, roff, foff, rows, width, shift, A, S, res[r], Gd, L,
                            epoch, pushed=True)
        for r in range(world):
            ops.peer_gather(bases, world, r, 0, foff, rows, width, res[r], epoch)
        torch.cuda.synchronize()
        for r in range(world):
            got = res[r].cpu().numpy()
            assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), f"rank {r} epoch {epoch}"
    assert _native.device_error(dev.index or 0) == 0


@pytest.mark.parametrize("world,rows,width,k", [(2, 130, 512, 512), (4, 77, 264, 256),
                                                (8, 99, 1024, 256)])
def test_peer_transport_copy_engine_bit_exact(cuda_device, oracle, world, rows, width, k):
    """The copy-engine exchange: each emulated rank pulls the other ranks' rows of its
    block into its staging slots (h3_copy_async), reduces them with its own rows into its
    residual rows and its own final area (h3_peer_reduce_staged), then pulls the other
    ranks' finished rows into its residual.  The flags h3_peer_signal waits for are set
    before it runs, so no kernel waits for another."""
    from h3tp import _native, ops, transport
    rng = np.random.default_rng(world + 80)
    shift = transport.shift_for(k, world)
    qs = [rng.integers(-128, 128, size=(rows, k), dtype=np.int8) for _ in range(world)]
    ws = [rng.integers(-127, 128, size=(width, k), dtype=np.int8) for _ in range(world)]
    enc = np.stack([oracle.fp16_encode(oracle.int8_gemm(q, w), shift) for q, w in zip(qs, ws)])
    a = rng.uniform(1e-4, 1e-2, size=rows).astype(np.float32)
    s = rng.uniform(1e-5, 1e-4, size=width).astype(np.float32)
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((3, width)).astype(np.float32)
    labels = rng.integers(0, 3, size=rows).astype(np.int32)
    ref = X.copy()
    oracle.row_reduce_finish(enc, shift, a, s, out="residual", residual=ref, gate=G, labels=labels)

    dev = cuda_device
    per = -(-rows // world)
    pitch = width * 2
    roff = FLAGS
    foff = roff + _region(rows, width)
    soff = foff + _region(rows, width)
    nbytes = soff + _region(world * per, width)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(world)]
    bases = [b.data_ptr() for b in bufs]
    A, S = torch.from_numpy(a).to(dev), torch.from_numpy(s).to(dev)
    Gd, L = torch.from_numpy(G).to(dev), torch.from_numpy(labels).to(dev)
    qd = [torch.from_numpy(q).to(dev) for q in qs]
    wd = [torch.from_numpy(w).to(dev) for w in ws]
    res = [torch.from_numpy(X.copy()).to(dev) for _ in range(world)]
    blocks = [(min(rows, r * per), min(rows, (r + 1) * per)) for r in range(world)]
    for epoch in (1, 2):
        for r in range(world):
            res[r].copy_(torch.from_numpy(X))
            part = bufs[r][roff:roff + rows * pitch].view(torch.float16).view(rows, width)
            ops.int8_gemm_row_encode(qd[r], wd[r], shift, out=part)
        for b in bufs:
            _set(b, READY, range(world), epoch)
        for r in range(world):
            ops.peer_signal(bases, world, r, 0, 0, epoch, True, res[r])
            b0, b1 = blocks[r]
            for k_ in range(1, world):
                w = (r + k_) % world
                ops.copy_async(bases[r] + soff + w * per * pitch, bases[w] + roff + b0 * pitch,
                               (b1 - b0) * pitch, res[r])
        for r in range(world):
            b0, _ = blocks[r]
            ops.peer_reduce_staged(bases, world, r, 0, soff, roff + b0 * pitch, foff, rows, width,
                                   shift, A, S, res[r], Gd, L, epoch)
        for r in range(world):
            ops.peer_signal(bases, world, r, 0, 1, epoch, False, res[r])
            for k_ in range(1, world):
                w = (r + k_) % world
                w0, w1 = blocks[w]
                ops.copy_async(res[r].data_ptr() + w0 * pitch, bases[w] + foff + w0 * pitch,
                               (w1 - w0) * pitch, res[r])
        torch.cuda.synchronize()
        for r in range(world):
            got = res[r].cpu().numpy()
            assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), f"rank {r} epoch {epoch}"
    assert _native.device_error(dev.index or 0) == 0


@pytest.mark.parametrize("world,rows,width,k", [(2, 130, 512, 512), (8, 99, 1024, 256)])
def test_peer_transport_packed_int8_bit_exact(cuda_device, oracle, world, rows, width, k):
    """The same exchange with the packed INT8 payload ('int8_gather'): the row GEMM packs
    in its epilogue, h3_peer_reduce_int8 reconstructs in rank order."""
    from h3tp import _native, ops
    rng = np.random.default_rng(world + 100)
    qs = [rng.integers(-128, 128, size=(rows, k), dtype=np.int8) for _ in range(world)]
    ws = [rng.integers(-127, 128, size=(width, k), dtype=np.int8) for _ in range(world)]
    packed = np.stack([oracle.pack8(oracle.int8_gemm(q, w)) for q, w in zip(qs, ws)])
    restored = oracle.unpack8_restore(packed, width)
    a = rng.uniform(1e-6, 1e-4, size=rows).astype(np.float32)
    s = rng.uniform(1e-5, 1e-4, size=width).astype(np.float32)
    X = rng.standard_normal((rows, width)).astype(np.float16)
    G = rng.standard_normal((3, width)).astype(np.float32)
    labels = rng.integers(0, 3, size=rows).astype(np.int32)
    ref = X.copy()
    oracle.dequantize_i32(restored, a, s, out="residual", residual=ref, gate=G, labels=labels)

    dev = cuda_device
    bufs, poff, foff = _buffers(dev, world, rows, width)
    bases = [b.data_ptr() for b in bufs]
    pitch = ops.pack8_pitch(width)
    A, S = torch.from_numpy(a).to(dev), torch.from_numpy(s).to(dev)
    Gd, L = torch.from_numpy(G).to(dev), torch.from_numpy(labels).to(dev)
    res = [torch.from_numpy(X.copy()).to(dev) for _ in range(world)]
    for r in range(world):
        part = bufs[r][poff:poff + rows * pitch].view(rows, pitch)
        ops.int8_gemm_row_pack8(torch.from_numpy(qs[r]).to(dev), torch.from_numpy(ws[r]).to(dev),
                                out=part)
    torch.cuda.synchronize()
    for r in range(world):
        got = bufs[r][poff:poff + rows * pitch].view(rows, pitch).cpu().numpy()
        assert np.array_equal(got, packed[r]), r
    for b in bufs:
        _set(b, READY, range(world), 1)
    for r in range(world):
        ops.peer_reduce_int8(bases, world, r, 0, poff, foff, rows, width, A, S, res[r], Gd, L, 1)
    for r in range(world):
        ops.peer_gather(bases, world, r, 0, foff, rows, width, res[r], 1)
    torch.cuda.synchronize()
    for r in range(world):
        got = res[r].cpu().numpy()
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), f"rank {r}"
    assert _native.device_error(dev.index or 0) == 0


def test_peer_wait_gives_up_with_timeout_status(cuda_device):
    """Rank 1 never signals: the reduce gives up after its bounded wait, records
    H3_ERR_TIMEOUT, publishes no done flag, and the gather gives up too."""
    from h3tp import _native, ops
    dev = cuda_device
    rows, width = 16, 256
    bufs, roff, foff = _buffers(dev, 2, rows, width)
    bases = [b.data_ptr() for b in bufs]
    res = torch.zeros((rows, width), dtype=torch.float16, device=dev)
    A = torch.ones(rows, dtype=torch.float32, device=dev)
    S = torch.ones(width, dtype=torch.float32, device=dev)
    assert _native.device_error(dev.index or 0) == 0
    ops.peer_reduce(bases, 2, 0, 0, roff, foff, rows, width, 0, A, S, res, None, None, 1)
    assert _native.device_error(dev.index or 0) == _native.H3_ERR_TIMEOUT
    assert int(bufs[1][:FLAGS].view(torch.int32)[DONE // 4]) == 0
    ops.peer_gather(bases, 2, 0, 0, foff, rows, width, res, 1)
    assert _native.device_error(dev.index or 0) == _native.H3_ERR_TIMEOUT
    assert _native.device_error(dev.index or 0) == 0  # reading clears it


def test_recorded_failure_reaches_the_next_forward_without_a_sync(cuda_device):
    """A bounded wait that gives up (rank 1 never signals) records H3_ERR_TIMEOUT in
    the host-mapped error word: h3_device_error_peek sees it without synchronising or
    clearing, the next module forward on that GPU raises H3Error, and once
    h3_device_error has read and cleared the word the forward runs again."""
    import time
    from h3tp import _native, ops
    from h3tp.tp_dit import ColumnParallelLinearINT8
    dev = cuda_device
    idx = dev.index or 0
    rows, width = 16, 256
    bufs, roff, foff = _buffers(dev, 2, rows, width)
    bases = [b.data_ptr() for b in bufs]
    res = torch.zeros((rows, width), dtype=torch.float16, device=dev)
    A = torch.ones(rows, dtype=torch.float32, device=dev)
    S = torch.ones(width, dtype=torch.float32, device=dev)
    assert _native.device_error(idx) == 0
    assert _native.device_error_peek(idx) == 0
    ops.peer_reduce(bases, 2, 0, 0, roff, foff, rows, width, 0, A, S, res, None, None, 1)
    deadline = time.time() + 30
    while _native.device_error_peek(idx) == 0 and time.time() < deadline:
        time.sleep(0.05)  # the word is read from host memory while the kernel waits
    assert _native.device_error_peek(idx) == _native.H3_ERR_TIMEOUT
    mod = ColumnParallelLinearINT8(256, 256, 0, 1, device=dev)
    mod.weight.data.fill_(1)
    mod.weight_scale.data.fill_(1e-3)
    x = torch.ones((4, 256), dtype=torch.float16, device=dev)
    with pytest.raises(_native.H3Error):
        with torch.no_grad():
            mod(x)
    assert _native.device_error(idx) == _native.H3_ERR_TIMEOUT  # synchronises, clears
    assert _native.device_error_peek(idx) == 0
    with torch.no_grad():
        y = mod(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_peer_rejects_bad_geometry(cuda_device):
    from h3tp import ops
    dev = cuda_device
    bufs, roff, foff = _buffers(dev, 2, 4, 256)
    bases = [b.data_ptr() for b in bufs]
    A = torch.ones(4, dtype=torch.float32, device=dev)
    with pytest.raises(ValueError):   # world 3 is not a TP size of the path
        ops.peer_reduce(bases + [bases[0]], 3, 0, 0, roff, foff, 4, 256, 0, A,
                        torch.ones(256, device=dev), torch.zeros((4, 256), dtype=torch.float16,
                                                                 device=dev))
    with pytest.raises(ValueError):   # width not a multiple of 8
        ops.peer_gather(bases, 2, 0, 0, foff, 4, 252, torch.zeros((4, 252), dtype=torch.float16,
                                                                   device=dev))
    with pytest.raises(ValueError):   # rows wider than the peer producer stages
        ops.swiglu_rotate_quantize_peer(
            torch.zeros((1, 2 * (ops.PEER_PRODUCER_MAX_WIDTH + 256)), dtype=torch.float16,
                        device=dev), bases, 2, 0, FLAGS, 1)


# ----------------------------------------------------------------------------
# FC2 producer with the row maxima exchanged over peer memory
# ----------------------------------------------------------------------------
def _producer_input(rng, kind, rows, width, special):
    if kind == "gateup_f16":
        g = rng.standard_normal((rows, width)).astype(np.float32)
        u = rng.standard_normal((rows, width)).astype(np.float32)
        g[::5] *= 40.0  # gates past the packed SiLU's range
        x = [g, u]
    else:
        x = [(rng.standard_normal((rows, width)) * 0.7).astype(np.float32)]
    if special:  # a NaN row, an inf row, a zero row
        x[0][0, 5] = np.nan
        x[0][1, 7] = np.inf
        x[0][2, :] = 0.0
    dtype = np.float32 if kind == "act_f32" else np.float16
    return np.concatenate(x, 1).astype(dtype)


def _slots(maxima, epoch):
    """u64 slots [rows][world] = (epoch << 32) | float bits, as every rank publishes."""
    bits = np.stack(maxima, 1).astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((np.uint64(epoch) << np.uint64(32)) | bits).view(np.int64)


@pytest.mark.parametrize("world,rows,width,kind", [(2, 37, 1024, "gateup_f16"),
                                                   (4, 300, 7168, "act_f32"),
                                                   (8, 64, 2048, "act_f16")])
def test_peer_producer_bit_exact(cuda_device, oracle, world, rows, width, kind):
    """Each emulated rank's slots hold every rank's row maximum (the oracle's) before
    its kernel runs, so no kernel waits for another; the codes and scales must equal
    the oracle's quantisation with the maximum over ranks, for two epochs in a row."""
    from h3tp import _native, ops
    rng = np.random.default_rng(world * 7 + width)
    xs = [_producer_input(rng, kind, rows, width, special=(r == 0)) for r in range(world)]
    rot = [oracle.fc2_rotate(x, kind) for x in xs]
    gmax = np.max(np.stack([m for _, m in rot]), 0)
    dev = cuda_device
    bufs = [torch.zeros(256 + rows * world * 8, dtype=torch.uint8, device=dev)
            for _ in range(world)]
    bases = [b.data_ptr() for b in bufs]
    xd = [torch.from_numpy(x).to(dev) for x in xs]
    for epoch in (1, 2):
        slots = torch.from_numpy(_slots([m for _, m in rot], epoch)).to(dev)
        for b in bufs:
            b[256:].view(torch.int64).view(rows, world).copy_(slots)
        for r in range(world):
            q, s, m = ops.swiglu_rotate_quantize_peer(xd[r], bases, world, r, 256, epoch, kind,
                                                      want_max=True)
            q_ref, s_ref = oracle.row_quantize(rot[r][0], gmax)
            got = q.cpu().numpy()
            assert np.array_equal(got, q_ref), f"rank {r} epoch {epoch}"
            assert np.array_equal(s.cpu().numpy().ravel().view(np.uint32), s_ref.view(np.uint32))
            assert np.array_equal(m.cpu().numpy().ravel().view(np.uint32), gmax.view(np.uint32))
    assert _native.device_error(dev.index or 0) == 0


def test_peer_producer_wait_gives_up(cuda_device, oracle):
    """Rank 1 never publishes: rank 0's CTAs give up after their bounded wait, record
    H3_ERR_TIMEOUT and quantise with the local maxima."""
    from h3tp import _native, ops
    dev = cuda_device
    rows, width = 6, 512
    x = _producer_input(np.random.default_rng(3), "gateup_f16", rows, width, special=False)
    R, m_loc = oracle.fc2_rotate(x, "gateup_f16")
    bufs = [torch.zeros(256 + rows * 2 * 8, dtype=torch.uint8, device=dev) for _ in range(2)]
    assert _native.device_error(dev.index or 0) == 0
    q, s, _ = ops.swiglu_rotate_quantize_peer(torch.from_numpy(x).to(dev),
                                              [b.data_ptr() for b in bufs], 2, 0, 256, 1)
    torch.cuda.synchronize()
    assert _native.device_error(dev.index or 0) == _native.H3_ERR_TIMEOUT
    q_ref, s_ref = oracle.row_quantize(R, m_loc)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    # rank 0 published its maxima into rank 1's slots
    pub = bufs[1][256:].view(torch.int64).view(rows, 2)[:, 0].cpu().numpy().view(np.uint64)
    assert (pub >> np.uint64(32) == 1).all()
    assert np.array_equal((pub & np.uint64(0xffffffff)).astype(np.uint32), m_loc.view(np.uint32))
