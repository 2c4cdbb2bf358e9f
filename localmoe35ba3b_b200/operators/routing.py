"""Route planner with the reference's CPU interface (replaces
qwen35_deploy/operators/routing.py:5-20).

The reference takes CPU ids and returns CPU ``positions [2, routes]`` and a
list of ``(expert, start, stop)`` segments.  Here the ids are copied to the
current CUDA device, the stable sort runs in the routing kernel, and the
results are copied back -- same values, same validation errors.
"""
import torch

from ..runtime import gpu_routes


def plan_routes(ids, experts):
    if ids.device.type != 'cpu' or ids.ndim != 2 or ids.numel() == 0:
        raise ValueError('Expected nonempty CPU [tokens,top_k] IDs')
    if int(ids.min()) < 0 or int(ids.max()) >= experts:
        raise ValueError('Out-of-range expert ID')
    dev = torch.device('cuda', torch.cuda.current_device())
    d = ids.to(dev, dtype=torch.int64).contiguous()
    top = ids.shape[1]
    pos, table, ordered, slots = gpu_routes.plan(d, experts, 1)
    # pos holds original // top; recover the flat order from ordered/slots
    flat = torch.empty(ids.numel(), dtype=torch.int64, device=dev)
    tok = torch.arange(ids.shape[0], device=dev)[:, None] * top
    flat.scatter_(0, ordered.reshape(-1), (tok + slots).reshape(-1))
    order = flat.cpu()
    counts = torch.bincount(ids.reshape(-1), minlength=experts).tolist()
    positions = torch.stack((order // top, order % top))
    segments = []
    start = 0
    for e, c in enumerate(counts):
        if c:
            segments.append((e, start, start + c))
            start += c
    return positions, segments
