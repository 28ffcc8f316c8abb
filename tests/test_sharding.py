"""Frame sharding across ranks (ml-video-denoiser_b200/sharding.py): segments
partition the sequence, temporal windows follow the reference's edge
replication, the halo covers every window, and sharded outputs equal the
single-rank outputs. The N > 1 logic runs as gloo ranks on the CPU; the GPU
test runs both ranks' segments through the real engine one after the other."""
import importlib
import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def S(pkg):
    return importlib.import_module(pkg.__name__ + ".sharding")


@pytest.mark.parametrize("n,world", [(10, 1), (10, 3), (7, 8), (240, 8), (1, 2), (0, 4)])
def test_segments_partition_the_sequence(S, n, world):
    segs = [S.segment(n, world, r) for r in range(world)]
    assert segs[0][0] == 0 and segs[-1][1] == n
    for (s0, e0), (s1, e1) in zip(segs, segs[1:]):
        assert e0 == s1
    sizes = [e - s for s, e in segs]
    assert max(sizes) - min(sizes) <= 1


def test_window_matches_reference_edge_replication(S):
    # training/infer.py:277-281: clamp(centre + offset, 0, n - 1) for offset in [-r, r]
    n = 6
    for T in (1, 3, 5):
        r = T // 2
        for c in range(n):
            assert S.window(c, T, n) == [min(max(c + o, 0), n - 1) for o in range(-r, r + 1)]
    with pytest.raises(ValueError):
        S.window(0, 4, n)


@pytest.mark.parametrize("n,world,T", [(20, 4, 5), (9, 2, 3), (5, 8, 5), (30, 3, 1)])
def test_halo_covers_every_window(S, n, world, T):
    for p in S.plan(n, world, T):
        s, e = p["segment"]
        assert len(p["windows"]) == e - s
        for i, win in zip(range(s, e), p["windows"]):
            assert [p["loads"][k] for k in win] == S.window(i, T, n)
        if s < e:
            assert len(p["loads"]) <= (e - s) + 2 * (T // 2)


def _fake_denoise(frames, idx):
    # a deterministic stand-in for the model: weighted mean over the window
    w = np.arange(1, len(idx) + 1, dtype=np.float64)
    return sum(wi * frames[i] for wi, i in zip(w, idx)) / w.sum()


def _rank_main(rank, world, n, T, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        here = os.path.dirname(os.path.abspath(__file__))
        import sys

        sys.path.insert(0, os.path.dirname(here))
        from __graft_entry__ import load_package

        S = importlib.import_module(load_package().__name__ + ".sharding")
        frames = [np.full((2, 3), float(i * i)) for i in range(n)]
        s, e = S.segment(n, world, rank)
        loads = S.needed_frames(n, world, rank, T)
        local = {f: frames[f] for f in loads}  # only what this rank loaded
        outs = {i: _fake_denoise(local, S.window(i, T, n)) for i in range(s, e)}
        gathered = [None] * world
        dist.all_gather_object(gathered, outs)  # test-side check only
        if rank == 0:
            merged = {}
            for g in gathered:
                merged.update(g)
            ref = {i: _fake_denoise(frames, S.window(i, T, n)) for i in range(n)}
            ok = sorted(merged) == list(range(n)) and all(np.array_equal(merged[i], ref[i]) for i in ref)
            q.put(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 5])
def test_gloo_two_ranks_equal_single_rank(T):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000) + T
    procs = [ctx.Process(target=_rank_main, args=(r, 2, 11, T, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=10) is True


@pytest.mark.gpu
def test_sharded_temporal_engine_equals_single_rank(pkg, S, tmp_path):
    import torch

    synth = importlib.import_module(pkg.__name__ + ".synth")
    cfg = synth.NAFConfig(base_channels=8, enc_blocks=(1, 1), middle_blocks=1, dec_blocks=(1, 1))
    path, _ = synth.make_model_dir(str(tmp_path), cfg, 3, "py", 3, True)
    m = pkg.Model(path)
    n, H, W = 7, 36, 44
    rng = np.random.default_rng(5)
    seq = [torch.from_numpy(rng.uniform(0, 1, (3, H, W)).astype(np.float16)).cuda() for _ in range(n)]
    whole = {i: y.clone() for i, y in S.denoise_segment(m, lambda i: seq[i], n, 1, 0, 3, cache=False)}
    parts = {}
    for r in range(3):
        parts.update({i: y.clone() for i, y in S.denoise_segment(m, lambda i: seq[i], n, 3, r, 3, cache=False)})
    torch.cuda.synchronize()
    assert sorted(parts) == list(range(n))
    for i in range(n):
        assert torch.equal(parts[i], whole[i]), i
    # the frame cache (each frame encoded once) gives the same frames: the
    # per-frame encoder pools over one image instead of a batch of T, so the
    # pool sums group differently and agree to FP32 rounding
    cached = {}
    for r in range(3):
        cached.update({i: y.clone() for i, y in S.denoise_segment(m, lambda i: seq[i], n, 3, r, 3, cache=True)})
    m.sync()
    for i in range(n):
        assert float((cached[i].float() - whole[i].float()).abs().max()) <= 2e-3, i


@pytest.mark.gpu
@pytest.mark.parametrize("kind,T", [("legacy", 3), ("py", 5)])
def test_frame_cache_matches_clip_forward(pkg, S, tmp_path, kind, T):
    import torch

    synth = importlib.import_module(pkg.__name__ + ".synth")
    cfg = synth.NAFConfig(base_channels=8, enc_blocks=(1, 1), middle_blocks=1, dec_blocks=(1, 1))
    path, _ = synth.make_model_dir(str(tmp_path), cfg, 4, kind, T, True)
    m = pkg.Model(path)
    n, H, W = 9, 30, 42
    rng = np.random.default_rng(6)
    seq = [torch.from_numpy(rng.uniform(0, 1, (3, H, W)).astype(np.float16)).cuda() for _ in range(n)]
    ref = {i: y.clone() for i, y in S.denoise_segment(m, lambda i: seq[i], n, 1, 0, T, cache=False)}
    got = {i: y.clone() for i, y in S.denoise_segment(m, lambda i: seq[i], n, 1, 0, T, cache=True)}
    m.sync()
    for i in range(n):
        assert float((got[i].float() - ref[i].float()).abs().max()) <= 2e-3, i
    with pytest.raises(pkg.InvalidArgumentError):
        m.encode_frame(seq[0].unsqueeze(0), T)


# ---------------------------------------------------------------------------
# Clip coordinator: a worker that dies or fails mid-segment (host only)
# ---------------------------------------------------------------------------

def _coord_main(rank, world, n, T, port, out_dir, fail_rank, fail_after, mode):
    import torch.distributed as dist

    from __graft_entry__ import load_package

    S = importlib.import_module(load_package().__name__ + ".sharding")
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=60))
    frames = [np.full((2, 3), float(i), np.float64) + np.arange(6).reshape(2, 3) * 0.01 for i in range(n)]
    coord = S.ClipCoordinator(store, rank, world, n, heartbeat_s=0.05, dead_after_s=0.6, poll_s=0.02)
    count = [0]

    def process_range(s, e, on_frame):
        for i in range(s, e):
            if rank == fail_rank and count[0] == fail_after:
                if mode == "exit":
                    os._exit(3)  # the process vanishes: no flag, the heartbeat stops
                raise RuntimeError("simulated worker failure")
            y = _fake_denoise(frames, S.window(i, T, n))
            np.save(os.path.join(out_dir, f"f{i:03d}_r{rank}.npy"), y)
            count[0] += 1
            on_frame(i)

    try:
        coord.run(process_range)
    except RuntimeError:
        pass  # reported to rank 0 through the store
    if rank == 0:
        with open(os.path.join(out_dir, "requeued.txt"), "w") as fh:
            fh.write(repr(coord.requeued()))
        # keep the store up until the others have seen `finished`
        import time
        time.sleep(0.5)


@pytest.mark.parametrize("mode", ["exit", "raise"])
def test_coordinator_requeues_a_failed_segment(pkg, tmp_path, mode):
    """Three CPU ranks share a 12-frame, T = 3 clip; rank 1 fails after one
    frame of its segment [4, 8), by vanishing or by raising. Rank 0 declares
    it dead and re-queues frames 5-7 to a live rank; every frame comes out
    exactly as in a single-rank run."""
    import multiprocessing as mp
    import socket

    S = importlib.import_module(pkg.__name__ + ".sharding")
    n, T, world = 12, 3, 3
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_coord_main, args=(r, world, n, T, port, str(tmp_path), 1, 1, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in procs)
    assert procs[0].exitcode == 0 and procs[2].exitcode == 0
    requeued = __import__("ast").literal_eval((tmp_path / "requeued.txt").read_text())
    assert len(requeued) == 1 and requeued[0][:2] == (5, 8) and requeued[0][2] in (0, 2)
    frames = [np.full((2, 3), float(i), np.float64) + np.arange(6).reshape(2, 3) * 0.01 for i in range(n)]
    for i in range(n):
        outs = sorted(tmp_path.glob(f"f{i:03d}_r*.npy"))
        assert outs, f"frame {i} missing"
        want = _fake_denoise(frames, S.window(i, T, n))
        for o in outs:
            assert np.array_equal(np.load(o), want)
    assert not list(tmp_path.glob("f00[5-7]_r1.npy"))  # rank 1 never finished them
