"""Frame sharding of a sequence across GPUs (one process per GPU).

Frames are independent for the spatial model, so rank r of W denoises the
contiguous segment ``segment(n, W, r)`` with no data exchange. The temporal
model needs, for output frame i, the window of T frames centred on i with
edge replication (``window``: cli/main.cc:163-174 and training/infer.py:
277-281 of the reference clamp ``i + t - T//2`` to ``[0, n-1]``), so a rank
also loads the ``T//2`` frames on each side of its segment (the halo) and
recomputes their encoder features; outputs are identical to a single-GPU
run. There is no collective on the data path.
"""
from __future__ import annotations


def segment(n_frames: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of the frames rank `rank` of `world` denoises: contiguous,
    sizes differing by at most one, earlier ranks taking the extra frames."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_frames < 0:
        raise ValueError("negative frame count")
    base, extra = divmod(n_frames, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def window(center: int, num_frames: int, n_frames: int) -> list[int]:
    """Frame indices of the temporal window of output frame `center`."""
    if num_frames <= 0 or num_frames % 2 == 0:
        raise ValueError("num_frames must be a positive odd number")
    if not 0 <= center < n_frames:
        raise ValueError("center outside the sequence")
    r = num_frames // 2
    return [min(max(center + t - r, 0), n_frames - 1) for t in range(num_frames)]


def needed_frames(n_frames: int, world: int, rank: int, num_frames: int = 1) -> list[int]:
    """Sorted frame indices rank `rank` must load: its segment plus the
    clamped halo its temporal windows reach (just the segment when
    num_frames == 1)."""
    s, e = segment(n_frames, world, rank)
    if s == e:
        return []
    r = num_frames // 2
    return list(range(max(0, s - r), min(n_frames, e + r)))


def plan(n_frames: int, world: int, num_frames: int = 1) -> list[dict]:
    """Per-rank work plan: segment, frames to load, and per output frame its
    window as positions into the loaded list."""
    out = []
    for rank in range(world):
        s, e = segment(n_frames, world, rank)
        loads = needed_frames(n_frames, world, rank, num_frames)
        pos = {f: i for i, f in enumerate(loads)}
        wins = [[pos[f] for f in window(i, num_frames, n_frames)] for i in range(s, e)] if num_frames > 1 else \
            [[pos[i]] for i in range(s, e)]
        out.append({"rank": rank, "segment": (s, e), "loads": loads, "windows": wins})
    return out


def denoise_segment(model, frames, n_frames: int, world: int, rank: int, num_frames: int = 1, stream=None,
                    cache: bool = True):
    """Denoise this rank's segment on its device (``denoise_range`` over
    ``segment(n_frames, world, rank)``).

    `model` is a ``Model`` (spatial when num_frames == 1, else temporal with
    that window); `frames(i)` returns frame i as a (C, H, W) FP16 CUDA tensor.
    Returns the list of (frame index, (3, H, W) output) for the segment."""
    s, e = segment(n_frames, world, rank)
    return denoise_range(model, frames, n_frames, s, e, num_frames, stream, cache)


def denoise_range(model, frames, n_frames: int, start: int, end: int, num_frames: int = 1, stream=None,
                  cache: bool = True, on_frame=None):
    """Denoise frames [start, end) of an n_frames sequence, loading the
    T//2 halo frames its windows reach. Returns [(frame index, output)];
    ``on_frame(i, y)``, when given, is called after each output.

    Temporal models use the engine's frame cache (``cache=True``): frame f is
    encoded once into slot f % T (distinct frames of one window never share a
    slot) and each output decodes its window from the slots, so the encoder
    runs once per loaded frame instead of T times per output. With
    ``cache=False`` every window is assembled as a (1, T, C, H, W) clip."""
    import torch

    s, e = start, end
    results = []

    def emit(i, y):
        results.append((i, y))
        if on_frame is not None:
            on_frame(i, y)

    if num_frames == 1:
        for i in range(s, e):
            emit(i, model(frames(i).unsqueeze(0).contiguous(), stream=stream)[0])
        return results
    if not cache:
        r = num_frames // 2
        held = {f: frames(f) for f in range(max(0, s - r), min(n_frames, e + r))}
        for i in range(s, e):
            x = torch.stack([held[f] for f in window(i, num_frames, n_frames)], dim=0).unsqueeze(0)
            emit(i, model(x.contiguous(), stream=stream)[0])
        return results
    T = num_frames
    in_slot = [-1] * T  # frame index held by each slot
    for i in range(s, e):
        win = window(i, T, n_frames)
        for f in win:
            if in_slot[f % T] != f:
                model.encode_frame(frames(f).unsqueeze(0).contiguous(), f % T, stream=stream)
                in_slot[f % T] = f
        emit(i, model.decode_window([f % T for f in win], frames(i).unsqueeze(0).contiguous(), stream=stream)[0])
    return results


# ---------------------------------------------------------------------------
# Clip coordinator with segment re-queue
# ---------------------------------------------------------------------------

class ClipCoordinator:
    """Runs one clip over `world` worker processes that share a key-value
    store (``torch.distributed.TCPStore``; rank 0 hosts it and coordinates).

    Work starts as the contiguous segments of ``segment``. Each worker
    processes its tasks frame by frame, marks every finished frame in the
    store and beats a heartbeat from a background thread. Rank 0 watches the
    heartbeats and the failure flags: a rank that reports a failure, or
    whose heartbeat is older than `dead_after_s`, is declared dead, and the
    unfinished frames of its tasks are re-queued as one new task for the live
    rank with the least remaining work. Frames are deterministic, so a frame
    finished twice (a worker declared dead while still alive stops at its
    next frame) gives the same output. Nothing here touches a GPU: the work
    is the caller's ``process_range(start, end, on_frame)``.

    Store keys: ``task/<k>`` = "start,end,rank", ``ntasks``, ``done/<i>``,
    ``hb/<rank>``, ``failed/<rank>``, ``dead/<rank>``, ``finished``."""

    def __init__(self, store, rank: int, world: int, n_frames: int, heartbeat_s: float = 0.2,
                 dead_after_s: float = 3.0, poll_s: float = 0.05):
        self.store, self.rank, self.world, self.n = store, rank, world, n_frames
        self.heartbeat_s, self.dead_after_s, self.poll_s = heartbeat_s, dead_after_s, poll_s

    # -- store helpers --
    def _get(self, key: str):
        return self.store.get(key).decode() if self.store.check([key]) else None

    def _task(self, k: int):
        s, e, r = (int(v) for v in self.store.get(f"task/{k}").decode().split(","))
        return s, e, r

    def _ntasks(self) -> int:
        return int(self.store.add("ntasks", 0))

    def _done(self, i: int) -> bool:
        return self.store.check([f"done/{i}"])

    def requeued(self) -> list:
        """Tasks created after the initial segments: [(start, end, rank)]."""
        return [self._task(k) for k in range(self.world, self._ntasks())]

    # -- roles --
    def _publish_plan(self):
        for r in range(self.world):
            s, e = segment(self.n, self.world, r)
            self.store.set(f"task/{r}", f"{s},{e},{r}")
        self.store.add("ntasks", self.world)

    def _beat(self, stop):
        import time

        while not stop.is_set():
            self.store.set(f"hb/{self.rank}", repr(time.time()))
            stop.wait(self.heartbeat_s)

    def _monitor(self, stop):
        import time

        start = time.time()
        dead = set()
        while not stop.is_set():
            if all(self._done(i) for i in range(self.n)):
                self.store.set("finished", "1")
                return
            now = time.time()
            for r in range(self.world):
                if r == self.rank or r in dead:
                    continue
                hb = self._get(f"hb/{r}")
                failed = self.store.check([f"failed/{r}"])
                stale = (now - float(hb)) > self.dead_after_s if hb else (now - start) > self.dead_after_s
                if failed or stale:
                    dead.add(r)
                    self.store.set(f"dead/{r}", "1")
                    self._requeue(r, dead)
            stop.wait(self.poll_s)

    def _requeue(self, r: int, dead: set):
        todo = []
        for k in range(self._ntasks()):
            s, e, owner = self._task(k)
            if owner == r:
                todo += [i for i in range(s, e) if not self._done(i)]
        if not todo:
            return
        live = [q for q in range(self.world) if q not in dead]
        load = {q: sum(1 for k in range(self._ntasks()) for i in range(*self._task(k)[:2])
                       if self._task(k)[2] == q and not self._done(i)) for q in live}
        target = min(live, key=lambda q: (load[q], q))
        # unfinished frames of a dead rank's tasks are a contiguous tail of
        # each task; re-queue them as contiguous runs
        runs, a = [], todo[0]
        for p, q in zip(todo, todo[1:] + [None]):
            if q != p + 1:
                runs.append((a, p + 1))
                a = q
        for s, e in runs:
            k = int(self.store.add("ntasks", 1)) - 1
            self.store.set(f"task/{k}", f"{s},{e},{target}")

    def run(self, process_range):
        """Work until the clip is finished; returns the frame indices this
        rank produced. process_range(start, end, on_frame) must call
        on_frame(i) after finishing frame i (and may raise to report a failure)."""
        import threading

        if self.rank == 0:
            self._publish_plan()
        else:
            self.store.wait(["ntasks"])
        stop = threading.Event()
        threads = [threading.Thread(target=self._beat, args=(stop,), daemon=True)]
        if self.rank == 0:
            threads.append(threading.Thread(target=self._monitor, args=(stop,), daemon=True))
        for t in threads:
            t.start()
        produced, started = [], set()

        class _Stop(Exception):
            pass

        def on_frame(i):
            self.store.set(f"done/{i}", str(self.rank))
            produced.append(i)
            if self.store.check([f"dead/{self.rank}"]):
                raise _Stop()

        try:
            while not self.store.check(["finished"]):
                mine = [k for k in range(self._ntasks()) if k not in started and self._task(k)[2] == self.rank]
                if not mine:
                    threading.Event().wait(self.poll_s)
                    continue
                for k in mine:
                    started.add(k)
                    s, e, _ = self._task(k)
                    try:
                        process_range(s, e, on_frame)
                    except _Stop:
                        return produced
                    except Exception:
                        self.store.set(f"failed/{self.rank}", "1")
                        raise
        finally:
            # On the normal path the monitor (rank 0) has already returned:
            # it sets `finished` once every frame is done. Rank 0 hosts the
            # store, so a failure of rank 0 itself ends the whole run.
            stop.set()
        return produced
