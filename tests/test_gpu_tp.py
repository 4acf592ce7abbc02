"""Tensor parallel inside one launch on two GPUs (ls_b200_tp_setup /
ls_b200_tp_connect): groups are sharded round-robin (leanstream_b200/tp.py),
each rank runs the same chained layers, and at the end of every layer the
ranks exchange their fp32 partial outputs over NVLink peer memory inside the
persistent kernel. Checked: both ranks hold identical outputs; a multi-layer
launch equals chained one-layer launches bit for bit; every layer equals the
oracle (sum of the ranks' partials in rank order, one fp16 rounding, the
residual) within the output tolerance. The IPC handles travel over a gloo
group on the host; the data path uses no NCCL. Skipped below two GPUs."""
import os
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

G, NGROUPS, LAYERS = 64, 24, 3
TOL = 2e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layers(H):
    from leanstream_b200.synthetic import make_layer

    Ls = [make_layer(500 + l, H, NGROUPS, G) for l in range(LAYERS)]
    sets = [np.sort(np.random.default_rng(70 + l).permutation(NGROUPS)[: 9 + 4 * l]) for l in range(LAYERS)]
    return Ls, sets


def _rank_main(rank, world, port, H, out_path):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    from gpu_harness import to_dev
    from leanstream_b200 import B200Backend, ExecutionQueue, tp
    from leanstream_b200 import _native as N

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Ls, sets = _layers(H)
        nloc = len(tp.local_groups(NGROUPS, rank, world))
        gb = G * 3 * H // 2
        be = B200Backend().configure(H, G, nloc, max_layers=LAYERS, cache_slots=nloc, physical_groups=nloc,
                                     timeout_us=2_000_000, rms_eps=1e-5)
        handle = be.tp_setup(rank, world)
        handles = [None] * world
        dist.all_gather_object(handles, handle)
        be.tp_connect(handles)
        keep, queues = [], []
        for l in range(LAYERS):
            rows = tp.rank_descriptors(sets[l], rank, world)
            q = ExecutionQueue(max(nloc, 1))
            q.reset(l + 1)
            if len(rows):
                q.write_descriptors(rows)
            q.prepare(len(rows))
            q.publish_all()
            q.activate()
            queues.append(q)
            packed = tp.shard_groups(Ls[l].packed.reshape(NGROUPS, gb), rank, world).reshape(-1)
            scales = tp.shard_groups(Ls[l].scales.reshape(NGROUPS, -1), rank, world).reshape(-1)
            keep += [to_dev(packed), to_dev(scales.view(np.int16), torch.float16)]
        x0 = to_dev(Ls[0].x.view(np.int16), torch.float16)

        def run(multi):
            xs = [x0.clone()] + [torch.zeros(H, dtype=torch.float16, device="cuda") for _ in range(LAYERS)]
            y = torch.zeros(H, dtype=torch.float16, device="cuda")
            y32 = torch.zeros(H, dtype=torch.float32, device="cuda")
            args = [be.layer_args(input=xs[l], output=y, cache=keep[2 * l], scales=keep[2 * l + 1], epoch=l + 1,
                                  queue=queues[l].view, mode=N.MODE_BATCH_COMPAT, layer=l, flags=N.NORM_INPUT,
                                  residual=xs[l], hidden_out=xs[l + 1], output_f32=y32) for l in range(LAYERS)]
            if multi:
                host = torch.frombuffer(bytearray(b"".join(be.encode_plan(a) for a in args)), dtype=torch.uint8)
                dev = host.cuda()
                be.launch_plans(dev, LAYERS, host.numpy().ctypes.data)
            else:
                for a in args:
                    be.launch(a)
            ev = torch.cuda.Event()
            ev.record()
            deadline = time.monotonic() + 20.0
            while not ev.query():
                assert time.monotonic() < deadline, "GPU work did not finish before the host deadline"
                time.sleep(0.001)
            torch.cuda.synchronize()
            st = be.status()
            assert st[N.STATUS_ERROR] == 0, st
            return [x.cpu().numpy().view(np.uint16).copy() for x in xs] + [
                y.cpu().numpy().view(np.uint16).copy(), y32.cpu().numpy().view(np.uint32).copy()]

        single = run(False)
        multi = run(True)
        dist.barrier()
        np.save(out_path.format(rank, 0), np.stack([a.astype(np.uint32) for a in single]))
        np.save(out_path.format(rank, 1), np.stack([a.astype(np.uint32) for a in multi]))
        be.close()
    finally:
        dist.destroy_process_group()


def _spawn(world, H, out, limit_s=240.0):
    import torch.multiprocessing as mp

    ctx = mp.start_processes(_rank_main, args=(world, _free_port(), H, out), nprocs=world, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + limit_s
    while not ctx.join(timeout=1.0):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            raise AssertionError("tensor-parallel ranks did not finish in time")


@pytest.mark.parametrize("H", [1024, 4096, 8192])
def test_two_gpu_exchange_matches_oracle(native_lib, cuda_device, tmp_path, H):
    import torch

    from leanstream_b200 import tp
    from leanstream_b200.synthetic import descriptors
    from oracle import oracle as O

    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "rank{}_{}.npy")
    _spawn(world, H, out)
    res = {(r, m): np.load(out.format(r, m)) for r in range(world) for m in range(2)}
    for m in range(2):
        assert np.array_equal(res[(0, m)], res[(1, m)]), "ranks must hold identical outputs"
    assert np.array_equal(res[(0, 0)], res[(0, 1)]), "multi-layer launch must equal chained launches"

    Ls, sets = _layers(H)
    gb = G * 3 * H // 2
    xs = [res[(0, 1)][l].astype(np.uint16).view(np.float16) for l in range(LAYERS + 1)]
    for l in range(LAYERS):
        x_l = xs[l]
        assert np.isfinite(x_l.astype(np.float32)).all()
        xin = O.rmsnorm(x_l, None, 1e-5)
        total = np.zeros(H, np.float32)
        for r in range(world):
            rows = tp.rank_descriptors(sets[l], r, world)
            if len(rows):
                packed = tp.shard_groups(Ls[l].packed.reshape(NGROUPS, gb), r, world).reshape(-1)
                scales = tp.shard_groups(Ls[l].scales.reshape(NGROUPS, -1), r, world).reshape(-1)
                _, y32, _ = O.mlp(H, G, xin, packed, scales, rows)
                total += y32
        ref = O.residual(x_l, total.astype(np.float16)).astype(np.float32)
        got = xs[l + 1].astype(np.float32)
        assert np.abs(got - ref).max() <= TOL * np.abs(ref).max() + 1e-3, (l, np.abs(got - ref).max())
        # and against the unsharded layer
        y_ref, _, _ = O.mlp(H, G, xin, Ls[l].packed, Ls[l].scales, descriptors(sets[l]))
        full = O.residual(x_l, y_ref).astype(np.float32)
        assert np.abs(got - full).max() <= TOL * np.abs(full).max() + 1e-3
    # the last layer's outputs: y = fp16(y32), x_L = fp16(x_{L-1} + y)
    y = res[(0, 1)][LAYERS + 1].astype(np.uint16).view(np.float16)
    y32 = res[(0, 1)][LAYERS + 2].astype(np.uint32).view(np.float32)
    assert np.array_equal(y, y32.astype(np.float16))
    assert np.array_equal(xs[LAYERS].view(np.uint16), O.residual(xs[LAYERS - 1], y).view(np.uint16))
