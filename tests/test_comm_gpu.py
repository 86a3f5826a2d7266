"""NVLink collective kernels.

* 1 GPU: a reduce whose peer flag is never set gives up after its budget, records the timeout in the
  device status word and leaves the context usable (pull reduce, push reduce and the skip agreement);
  the push reduce-scatter's index arithmetic on a world of one.
* 2 GPUs (one process each, NCCL only for rendezvous): packed bf16/fp32 gradients reduced by their
  owners equal the mean of the ranks' inputs; the parameter gather (pull) and the parameter push
  deliver the owners' values and refresh bf16 shadows; the fused top-k path reduces the kept entries;
  the trainer's p2p path tracks the NCCL path step for step.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda):
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    check_status()
    ptr, _ = E.sym_alloc(1 << 20)
    try:
        flags = torch.tensor([ptr], dtype=torch.int64, device=cuda)
        peers = torch.tensor([ptr], dtype=torch.int64, device=cuda)
        chunks = torch.tensor([[0, 1024]], dtype=torch.int64, device=cuda)
        out = torch.zeros(1024, device=cuda)
        t0 = time.time()
        E.comm_reduce(peers, flags, 0, 1, chunks, out, 0, 1.0, 4, 0.2)  # flag stays 0 < epoch 1
        torch.cuda.synchronize()
        dt = time.time() - t0
        assert check_status() == 4  # kErrTimeoutPeer
        assert 0.15 < dt < 5.0
        x = torch.randn(1000, device=cuda)  # context still healthy
        assert torch.isfinite((x @ x).reshape(1)).all()
    finally:
        E.sym_free(ptr)


def test_push_reduce_and_agree_time_out_and_context_survives(cuda):
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    check_status()
    ptr, _ = E.sym_alloc(1 << 20)
    try:
        chunks = torch.tensor([[0, 1024, 0, 0]], dtype=torch.int64, device=cuda)
        out = torch.zeros(1024, device=cuda)
        t0 = time.time()
        E.comm_reduce_local(ptr, ptr + (1 << 19), 1, 0, 1, 1024, chunks, out, 0, 1.0, 4, 0.2)  # flag stays 0
        torch.cuda.synchronize()
        assert check_status() == 4 and 0.15 < time.time() - t0 < 5.0
        skip = torch.zeros(1, dtype=torch.int32, device=cuda)
        E.comm_agree(ptr + (1 << 19), 1, 0, 1, skip, 0.2)
        torch.cuda.synchronize()
        assert check_status() == 4 and int(skip.item()) == 1  # a timed-out step is skipped
        x = torch.randn(1000, device=cuda)
        assert torch.isfinite((x @ x).reshape(1)).all()
    finally:
        E.sym_free(ptr)


@pytest.mark.parametrize("wire,code", [("fp32", 0), ("bf16", 1), ("fp16", 2)])
def test_push_reduce_scatter_world_of_one(cuda, wire, code):
    """pack_push -> signal_all -> reduce_local -> agree with this GPU as the only rank: two parameters
    with odd lengths at scattered slot offsets come back as scale * value; a NaN sets the skip word."""
    from bitresearch_b200.ops._ext import check_status, ext
    E = ext()
    check_status()
    wb = {0: 4, 1: 2, 2: 2}[code]
    slot = 4096
    rptr, _ = E.sym_alloc(slot * wb)
    fptr, _ = E.sym_alloc(2 * 8)
    try:
        grad = torch.randn(3000, device=cuda)
        # parameter a: flat [0, 1237) -> slot 2048; parameter b: flat [1248, 2990) -> slot 0
        chunks = torch.tensor([[0, 1237, 0, 2048], [1248, 1742, 0, 0]], dtype=torch.int64, device=cuda)
        peers = torch.tensor([rptr], dtype=torch.int64, device=cuda)
        fpeers = torch.tensor([fptr], dtype=torch.int64, device=cuda)
        bad = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = torch.zeros(3000, device=cuda)
        skip = torch.full((1,), 7, dtype=torch.int32, device=cuda)
        E.comm_pack_push(grad, peers, 0, slot, chunks, code, 0.5, bad, 0)
        E.comm_signal_all(fpeers, 0, 1, 1, bad)
        E.comm_reduce_local(rptr, fptr, 1, 1, 1, slot, chunks, out, code, 2.0, 0, 5.0)
        E.comm_agree(fptr, 1, 1, 1, skip, 5.0)
        torch.cuda.synchronize()
        assert check_status() == 0 and int(bad.item()) == 0 and int(skip.item()) == 0
        ref = grad * 0.5
        if code:
            ref = ref.to(torch.bfloat16 if code == 1 else torch.float16).float()
        ref = ref * 2.0
        for lo, hi in ((0, 1237), (1248, 2990)):
            torch.testing.assert_close(out[lo:hi], ref[lo:hi], rtol=0, atol=0)
        assert out[1237:1248].abs().max().item() == 0 and out[2990:].abs().max().item() == 0
        grad[5] = float("nan")  # next step: a non-finite gradient reaches the skip word
        bad.zero_()
        E.comm_pack_push(grad, peers, 0, slot, chunks, code, 0.5, bad, 0)
        E.comm_signal_all(fpeers, 0, 1, 2, bad)
        E.comm_agree(fptr, 1, 1, 2, skip, 5.0)
        torch.cuda.synchronize()
        assert int(bad.item()) == 1 and int(skip.item()) == 1 and check_status() == 0
    finally:
        E.sym_free(rptr)
        E.sym_free(fptr)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _to_numpy(x):
    """Results cross the queue as numpy arrays: a torch CPU tensor would travel as a shared-memory file
    descriptor that is gone once the child exits, which it may do before the parent reads it."""
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu()
        return ("__tensor__", (x.float() if x.dtype == torch.bfloat16 else x).numpy().copy(), str(x.dtype))
    if isinstance(x, dict):
        return {k: _to_numpy(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_to_numpy(v) for v in x)
    return x


def _to_torch(x):
    if isinstance(x, tuple) and len(x) == 3 and x[0] == "__tensor__":
        return torch.from_numpy(x[1])
    if isinstance(x, dict):
        return {k: _to_torch(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_to_torch(v) for v in x)
    return x


def _worker(rank, world, port, fn, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        q.put((rank, "ok", _to_numpy(fn(rank, world))))
    except BaseException:
        import traceback
        q.put((rank, "err", traceback.format_exc()))
    finally:
        try:
            torch.cuda.synchronize()
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fn, world=2, timeout=300):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, st, v = q.get(timeout=timeout)
            assert st == "ok", f"rank {r}:\n{v}"
            res[r] = _to_torch(v)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return [res[r] for r in range(world)]


def _reduce_gather(rank, world):
    from bitresearch_b200.ops._ext import check_status, ext
    from bitresearch_b200.parallel.comm import SymmetricBuffer
    E = ext()
    n = 40000
    out = {}
    for wire, code, nbytes in (("fp32", 0, 4), ("bf16", 1, 2)):
        send = SymmetricBuffer(n * nbytes)
        flags = SymmetricBuffer(64)
        g = torch.Generator(device="cpu").manual_seed(rank)
        src = torch.randn(n, generator=g).cuda()
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        E.comm_pack(src, send.ptr, code, 0, n, 0.5, bad)
        E.comm_signal(flags.ptr, 7)
        # rank r owns [r*n/2, (r+1)*n/2)
        half = n // 2
        chunks = torch.tensor([[rank * half, half]], dtype=torch.int64, device="cuda")
        red = torch.zeros(n, device="cuda")
        fp = torch.tensor(flags.peer_ptrs, dtype=torch.int64, device="cuda")
        E.comm_reduce(send.peers_dev, fp, 0, 7, chunks, red, code, 1.0 / world, 16, 10.0)
        torch.cuda.synchronize()
        out[wire] = (red[rank * half:(rank + 1) * half].cpu(), int(bad.item()), check_status())
        torch.distributed.barrier()
        send.close()
        flags.close()
    # gather: every rank pulls the other rank's half of a symmetric parameter buffer
    pbuf = SymmetricBuffer(n * 4)
    flags = SymmetricBuffer(64)
    local = E.sym_view(pbuf.ptr, n, 0, rank)
    local.copy_(torch.full((n,), float(rank + 1), device="cuda"))
    torch.cuda.synchronize()
    E.comm_signal(flags.ptr + 8, 3)
    other = 1 - rank
    shadow = torch.zeros(100, 200, dtype=torch.bfloat16, device="cuda")
    # the other half is a [100, 200] matrix with a bf16 shadow of row stride 200
    seg = torch.tensor([[other * (n // 2), n // 2, other, 200, 200, shadow.data_ptr(), 0]], dtype=torch.int64,
                       device="cuda")
    fp = torch.tensor(flags.peer_ptrs, dtype=torch.int64, device="cuda")
    E.comm_gather(pbuf.peers_dev, fp, 1, 3, seg, local, 8, 10.0)
    torch.cuda.synchronize()
    out["gather"] = (local.cpu(), shadow.float().cpu(), check_status())
    torch.distributed.barrier()
    pbuf.close()
    flags.close()
    return out


def test_p2p_reduce_and_gather_2gpu():
    res = _run(_reduce_gather)
    n, half = 40000, 20000
    srcs = [torch.randn(n, generator=torch.Generator().manual_seed(r)) for r in range(2)]
    mean = (srcs[0] + srcs[1]) * 0.5 * 0.5
    for r in range(2):
        red32, bad, st = res[r]["fp32"]
        assert st == 0 and bad == 0
        torch.testing.assert_close(red32, mean[r * half:(r + 1) * half], rtol=1e-6, atol=1e-6)
        red16, _, _ = res[r]["bf16"]
        torch.testing.assert_close(red16, mean[r * half:(r + 1) * half], rtol=1e-2, atol=1e-2)
        local, shadow, st = res[r]["gather"]
        assert st == 0
        other = 1 - r
        assert torch.all(local[other * half:(other + 1) * half] == other + 1)
        assert torch.all(local[r * half:(r + 1) * half] == r + 1)
        assert torch.all(shadow == other + 1)


def _push_rs(rank, world):
    """Two parameters owned by rank 0 and one by rank 1 (uneven ownership), two steps; on the second, rank 1
    has a NaN in a parameter rank 0 owns: rank 0's reduce sees it, and both ranks' skip words are set."""
    from bitresearch_b200.ops._ext import check_status, ext
    from bitresearch_b200.parallel.comm import SymmetricBuffer
    E = ext()
    out = {}
    for wire, code, wb in (("fp32", 0, 4), ("bf16", 1, 2)):
        slot = 3072  # rank 0 owns 1000 + 2000 (slots 0 and 1008), rank 1 owns 1500 (slot 0)
        recv = SymmetricBuffer(world * slot * wb)
        flags = SymmetricBuffer(2 * world * 8)
        rp = torch.tensor(recv.peer_ptrs, dtype=torch.int64, device="cuda")
        fp = torch.tensor(flags.peer_ptrs, dtype=torch.int64, device="cuda")
        # flat: a [0, 1000) owner 0 slot 0 | b [1008, 3008) owner 0 slot 1008 | c [3008, 4508) owner 1 slot 0
        table = [(0, 1000, 0, 0), (1008, 2000, 0, 1008), (3008, 1500, 1, 0)]
        allc = torch.tensor(table, dtype=torch.int64, device="cuda")
        mine = torch.tensor([t for t in table if t[2] == rank], dtype=torch.int64, device="cuda")
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        skip = torch.zeros(1, dtype=torch.int32, device="cuda")
        res = []
        for epoch in (1, 2):
            g = torch.randn(4508, generator=torch.Generator().manual_seed(10 * epoch + rank)).cuda()
            if epoch == 2 and rank == 1:
                g[1500] = float("nan")
            bad.zero_()
            red = torch.zeros(4508, device="cuda")
            E.comm_pack_push(g, rp, rank, slot, allc, code, 1.0, bad, 0)
            E.comm_signal_all(fp, rank, 1, epoch, bad)
            E.comm_reduce_local(recv.ptr, flags.ptr, world, 1, epoch, slot, mine, red, code, 1.0 / world, 0, 10.0)
            E.comm_agree(flags.ptr, world, 1, epoch, skip, 10.0)
            torch.cuda.synchronize()
            res.append((red.cpu(), int(skip.item()), check_status()))
            torch.distributed.barrier()
        out[wire] = res
        recv.close()
        flags.close()
    return out


def test_push_reduce_scatter_2gpu():
    res = _run(_push_rs)
    gs = {e: [torch.randn(4508, generator=torch.Generator().manual_seed(10 * e + r)) for r in range(2)] for e in (1, 2)}
    mean = (gs[1][0] + gs[1][1]) / 2
    own = {0: [(0, 1000), (1008, 3008)], 1: [(3008, 4508)]}
    for wire, tol in (("fp32", 1e-6), ("bf16", 1e-2)):
        for r in range(2):
            red, skip, st = res[r][wire][0]
            assert st == 0 and skip == 0
            for lo, hi in own[r]:
                torch.testing.assert_close(red[lo:hi], mean[lo:hi], rtol=tol, atol=tol)
            red2, skip2, st2 = res[r][wire][1]
            assert st2 == 0 and skip2 == 1  # both ranks agree to skip the step with rank 1's NaN
        assert torch.isnan(res[0][wire][1][0][1500])


def _push(rank, world):
    """Rank r owns half of a symmetric fp32 buffer; each pushes its half into the other and flags it;
    the shadow refresh waits for the flag and writes the bf16 shadow of the half it does not own."""
    from bitresearch_b200.ops._ext import check_status, ext
    from bitresearch_b200.parallel.comm import SymmetricBuffer
    E = ext()
    n, half = 40000, 20000
    pbuf = SymmetricBuffer(n * 4)
    pflags = SymmetricBuffer(world * 8)
    local = E.sym_view(pbuf.ptr, n, 0, rank)
    out = {}
    for epoch in (1, 2):  # two rounds: the flag protocol across steps
        local.copy_(torch.full((n,), 0.0, device="cuda"))
        local[rank * half:(rank + 1) * half] = float(10 * epoch + rank + 1)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        mine = torch.tensor([[rank * half, half]], dtype=torch.int64, device="cuda")
        E.comm_push(local, pbuf.peers_dev, rank, mine, 0)
        E.comm_signal_peers(pflags.peers_dev, rank, epoch)
        other = 1 - rank
        shadow = torch.zeros(100, 200, dtype=torch.bfloat16, device="cuda")
        seg = torch.tensor([[other * half, half, other, 200, 200, shadow.data_ptr(), 0]], dtype=torch.int64,
                           device="cuda")
        E.comm_shadow_refresh(local, pflags.ptr, world, rank, epoch, seg, 0, 10.0)
        torch.cuda.synchronize()
        out[epoch] = (local.cpu(), shadow.float().cpu(), check_status())
        torch.distributed.barrier()
    pbuf.close()
    pflags.close()
    return out


def test_parameter_push_and_shadow_refresh_2gpu():
    res = _run(_push)
    n, half = 40000, 20000
    for r in range(2):
        o = 1 - r
        for epoch in (1, 2):
            local, shadow, st = res[r][epoch]
            assert st == 0
            assert torch.all(local[r * half:(r + 1) * half] == 10 * epoch + r + 1)
            assert torch.all(local[o * half:(o + 1) * half] == 10 * epoch + o + 1)  # pushed by the owner
            assert torch.all(shadow == 10 * epoch + o + 1)


def _train(rank, world):
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    out = {}
    for comm in ("nccl", "p2p"):
        cfg = apply_overrides(preset("d512"), ["model.n_layer=2", "model.sequence_len=256", "model.vocab_size=1024",
                                               "device_batch=4", f"total_batch_tokens={4 * 256 * world}",
                                               "log_every=0", "results_tsv=", f"comm={comm}", "wire_dtype=fp32"])
        tr = Trainer(cfg, device=torch.device("cuda", rank), log=lambda m: None)
        tr.initialize()
        init = {n: p.detach().float().cpu().clone() for n, p in tr.model.named().items()}
        g = torch.Generator(device="cpu").manual_seed(100 + rank)
        losses, grads = [], None
        for step in range(3):
            x = torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda()
            y = torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda()
            losses.append(float(tr.train_step((x, y))))
            if step == 0:  # the mean gradient the optimizer consumed on the first step
                if comm == "nccl":
                    grads = {n: v.detach().float().cpu().clone() for n, v in tr.grad_views.items()}
                else:
                    grads = {n: tr.comm.red_views[n].detach().float().cpu().clone() for n in tr.comm.owned_names}
        torch.cuda.synchronize()  # the last parameter exchange runs on the comm stream
        out[comm] = (losses, {n: p.detach().float().cpu() for n, p in tr.model.named().items()}, grads, init)
        tr.destroy()
    return out


def test_p2p_trainer_matches_nccl_2gpu():
    """Same batches through the NCCL all-reduce path and the in-kernel NVLink path: ranks hold identical
    replicas, the mean gradients agree to fp32 accumulation-order noise, losses track, and after three
    steps each parameter's difference between the paths is small next to the distance it moved. (Muon
    matrices go through bf16 Newton-Schulz, batched over each rank's owned shard on the p2p path and
    over all matrices on the replicated path, so the two updates differ by bf16 rounding; AdamW with
    eps 1e-10 amplifies near-zero gradient differences into sign flips of single elements.)"""
    res = _run(_train)
    for n in res[0]["p2p"][1]:
        assert torch.equal(res[0]["p2p"][1][n], res[1]["p2p"][1][n]), n  # ranks hold identical replicas
    for r in range(2):
        ln, pn, gn, init = res[r]["nccl"]
        lp, pp, gp, _ = res[r]["p2p"]
        for a, b in zip(ln, lp):
            assert abs(a - b) < 2e-3 * abs(a)
        for n, g in gp.items():  # owned parameters of this rank
            ref = gn[n]
            err = (g - ref).abs().max().item()
            assert err <= 1e-4 * (ref.abs().max().item() + 1e-12), (n, err)
        for n in pn:
            moved = (pn[n] - init[n]).norm().item() + 1e-12
            diff = (pn[n] - pp[n]).norm().item()
            adam = not n.startswith("layer")
            assert diff <= (0.25 if adam else 0.1) * moved, (r, n, diff, moved)


def _device_skip(rank, world):
    """p2p trainer, 2 ranks: on the second step rank 1's gradient gets a NaN just before the first bucket is
    packed; both ranks must leave every parameter unchanged, learn of the skip one step later and keep
    identical replicas."""
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("d512"), ["model.n_layer=2", "model.sequence_len=256", "model.vocab_size=1024",
                                           "device_batch=4", f"total_batch_tokens={4 * 256 * world}",
                                           "log_every=0", "results_tsv=", "comm=p2p"])
    tr = Trainer(cfg, device=torch.device("cuda", rank), log=lambda m: None)
    tr.initialize()
    hook = tr.engine.bucket_hook
    state = {"poison": False}

    def poisoned(b, scale):
        if state["poison"] and b == 0:
            tr.flat_grad[tr.bucket_ranges[0][0]] = float("nan")
        hook(b, scale)

    tr.engine.bucket_hook = poisoned
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    batches = [(torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda(),
                torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda()) for _ in range(3)]
    tr.train_step(batches[0])
    torch.cuda.synchronize()
    before = {n: p.detach().float().cpu().clone() for n, p in tr.model.named().items()}
    state["poison"] = rank == 1
    tr.train_step(batches[1])
    torch.cuda.synchronize()
    after = {n: p.detach().float().cpu().clone() for n, p in tr.model.named().items()}
    skipped_late = tr.skipped
    state["poison"] = False
    tr.train_step(batches[2])  # polls the previous step's outcome
    torch.cuda.synchronize()
    tr.comm.poll(wait=True)
    final = {n: p.detach().float().cpu() for n, p in tr.model.named().items()}
    out = (before, after, skipped_late, tr.skipped, final)
    tr.destroy()
    return out


def test_device_side_skip_keeps_replicas_2gpu():
    res = _run(_device_skip)
    for r in range(2):
        before, after, skipped_late, skipped, _ = res[r]
        for n in before:
            assert torch.equal(before[n], after[n]), (r, n)  # the poisoned step changed nothing
        assert skipped == 1
    for n in res[0][4]:
        assert torch.equal(res[0][4][n], res[1][4][n]), n  # replicas identical after the next step
        assert torch.isfinite(res[0][4][n]).all(), n


def _overlap_forward(rank, world):
    """p2p trainer, 2 ranks: the forward queued right after a step (it waits per layer for the parameter
    exchange still running on the comm stream) gives bitwise the same per-token losses as the same forward
    run after a device synchronisation and a barrier."""
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("d512"), ["model.n_layer=4", "model.sequence_len=256", "model.vocab_size=1024",
                                           "device_batch=4", f"total_batch_tokens={4 * 256 * world}",
                                           "log_every=0", "results_tsv=", "comm=p2p"])
    tr = Trainer(cfg, device=torch.device("cuda", rank), log=lambda m: None)
    tr.initialize()
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    x = torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda()
    y = torch.randint(0, 1024, (4, 256), generator=g, dtype=torch.int32).cuda()
    out = []
    for _ in range(2):
        tr.train_step((x, y), sync=False)
        early = tr.engine.per_token_nats(x, y)  # queued behind the exchange, layer by layer
        torch.cuda.synchronize()
        torch.distributed.barrier()
        late = tr.engine.per_token_nats(x, y)
        torch.cuda.synchronize()
        out.append((early.cpu(), late.cpu()))
    tr.destroy()
    return out


def test_forward_overlapping_the_parameter_exchange_2gpu():
    res = _run(_overlap_forward)
    for r in range(2):
        for early, late in res[r]:
            assert torch.equal(early, late), (r, (early - late).abs().max().item())


@pytest.mark.parametrize("masking", [False, True])
def test_topk_select_momentum_modes_match_oracle(cuda, masking):
    """Three steps of threshold + select with a velocity, against an fp64 statement of the same update
    (reference form or the masked DGC form); entries within 1e-5 of the threshold may go either way."""
    from bitresearch_b200.ops._ext import ext
    E = ext()
    n, k, mu = 1 << 16, 0.01, 0.9
    gen = torch.Generator().manual_seed(3)
    err = torch.zeros(n, device="cuda")
    vel = torch.zeros(n, device="cuda")
    e64 = torch.zeros(n, dtype=torch.float64)
    v64 = torch.zeros(n, dtype=torch.float64)
    thr = torch.zeros(1, device="cuda")
    chunks = torch.tensor([[0, n, 0, 0]], dtype=torch.int64, device="cuda")
    for step in range(3):
        g = torch.randn(n, generator=gen)
        idx = torch.zeros(n, dtype=torch.int32, device="cuda")
        val = torch.zeros(n, dtype=torch.float16, device="cuda")
        cnt = torch.zeros(4, dtype=torch.int32, device="cuda")
        gd = g.cuda()
        E.topk_threshold(gd, err, vel, 0, n, 1.0, mu, 10000, k, 77 + step, masking, thr)
        E.topk_select(gd, err, vel, chunks, 1.0, mu, masking, thr, idx.data_ptr(), val.data_ptr(), cnt.data_ptr())
        torch.cuda.synchronize()
        t = float(thr.item())
        g64 = g.double()
        if masking:
            u = mu * v64 + g64
            a = e64 + u
        else:
            a = mu * v64 + (g64 + e64)
            u = a
        keep = a.abs() >= t
        sure = (a.abs() - t).abs() > 1e-5 * max(t, 1.0)
        m = int(cnt[0])
        sent = torch.zeros(n, dtype=torch.bool)
        sent[idx[:m].long().cpu()] = True
        assert m == int(sent.sum())  # no index twice
        assert torch.equal(sent[sure], keep[sure]), step
        assert 0.005 < keep.double().mean() < 0.02  # about k from a 10000-sample threshold
        torch.testing.assert_close(val[:m].float().cpu(), a[idx[:m].long().cpu()].half().float(), rtol=2e-3, atol=1e-4)
        # carry the kernel's own keep decision into the oracle (borderline entries included)
        e64 = torch.where(sent, torch.zeros_like(a), a)
        v64 = torch.where(sent, torch.zeros_like(u), u) if masking else u
        torch.testing.assert_close(err.cpu().double(), e64, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(vel.cpu().double(), v64, rtol=1e-5, atol=1e-5)


def _topk(rank, world):
    """One bucket of n elements; rank 0 owns the first half, rank 1 the second."""
    from bitresearch_b200.ops._ext import check_status, ext
    from bitresearch_b200.parallel.comm import SymmetricBuffer
    E = ext()
    n, half, k = 65536, 32768, 0.05
    g = torch.randn(n, generator=torch.Generator().manual_seed(10 + rank)).cuda()
    err = torch.zeros(n, device="cuda")
    thr = torch.zeros(1, device="cuda")
    idx = SymmetricBuffer(n * 4)
    val = SymmetricBuffer(n * 2)
    cnt = SymmetricBuffer(64)
    flags = SymmetricBuffer(64)
    # list regions: owner 0 at [0, half), owner 1 at [half, n); counters 0 and 1
    chunks = torch.tensor([[0, half, 0, 0], [half, half, half, 1]], dtype=torch.int64, device="cuda")
    E.topk_threshold(g, err, None, 0, n, 1.0, 0.0, 10000, k, 1234 + rank, False, thr)
    E.topk_select(g, err, None, chunks, 1.0, 0.0, False, thr, idx.ptr, val.ptr, cnt.ptr)
    E.comm_signal(flags.ptr, 5)
    peers = torch.tensor([[idx.peer_ptrs[r], val.peer_ptrs[r], cnt.peer_ptrs[r]] for r in range(world)],
                         dtype=torch.int64, device="cuda")
    fp = torch.tensor(flags.peer_ptrs, dtype=torch.int64, device="cuda")
    red = torch.zeros(n, device="cuda")
    E.topk_reduce(peers, fp, 0, 5, rank * half, rank, red, 1.0 / world, 16, 10.0)
    torch.cuda.synchronize()
    out = (g.cpu(), err.cpu(), float(thr.item()), red.cpu(), check_status())
    torch.distributed.barrier()
    for b in (idx, val, cnt, flags):
        b.close()
    return out


def test_topk_sparse_reduce_2gpu():
    res = _run(_topk)
    n, half = 65536, 32768
    kept = []
    for g, err, thr, _, st in res:
        assert st == 0
        keep = g.abs() >= thr
        assert 0.03 < keep.float().mean().item() < 0.07  # about k = 5% from a 10000-sample threshold
        torch.testing.assert_close(err, torch.where(keep, torch.zeros_like(g), g))  # residual = what was dropped
        kept.append(torch.where(keep, g, torch.zeros_like(g)).half().float())
    mean = (kept[0] + kept[1]) / 2
    for r, (_, _, _, red, _) in enumerate(res):
        sl = slice(r * half, (r + 1) * half)
        torch.testing.assert_close(red[sl], mean[sl], rtol=1e-3, atol=1e-3)
