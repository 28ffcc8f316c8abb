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
    """Denoise this rank's segment on its device.

    `model` is a ``Model`` (spatial when num_frames == 1, else temporal with
    that window); `frames(i)` returns frame i as a (C, H, W) FP16 CUDA tensor.
    Returns the list of (frame index, (3, H, W) output) for the segment.

    Temporal models use the engine's frame cache (``cache=True``): frame f is
    encoded once into slot f % T (distinct frames of one window never share a
    slot) and each output decodes its window from the slots, so the encoder
    runs once per loaded frame instead of T times per output. With
    ``cache=False`` every window is assembled as a (1, T, C, H, W) clip."""
    import torch

    s, e = segment(n_frames, world, rank)
    results = []
    if num_frames == 1:
        for i in range(s, e):
            y = model(frames(i).unsqueeze(0).contiguous(), stream=stream)
            results.append((i, y[0]))
        return results
    if not cache:
        loads = needed_frames(n_frames, world, rank, num_frames)
        held = {f: frames(f) for f in loads}
        for i in range(s, e):
            x = torch.stack([held[f] for f in window(i, num_frames, n_frames)], dim=0).unsqueeze(0)
            results.append((i, model(x.contiguous(), stream=stream)[0]))
        return results
    T = num_frames
    in_slot = [-1] * T  # frame index held by each slot
    for i in range(s, e):
        win = window(i, T, n_frames)
        for f in win:
            if in_slot[f % T] != f:
                model.encode_frame(frames(f).unsqueeze(0).contiguous(), f % T, stream=stream)
                in_slot[f % T] = f
        y = model.decode_window([f % T for f in win], frames(i).unsqueeze(0).contiguous(), stream=stream)
        results.append((i, y[0]))
    return results
