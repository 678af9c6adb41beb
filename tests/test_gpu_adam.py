"""The fused optimizer step (hds_adam_step, hds_b200.optim) against torch.optim.Adam(fused=True), the
reference training loop's optimizer (main.py:194), and against the oracle's Adam (the reference's
sh.cu:90-102 form) bit for bit: three steps over seven parameter groups of lengths that put segment
boundaries inside float4 chunks, plus buffers that start 4 bytes off 16-byte alignment (the element
path)."""
import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LRS = [0.00016 * 5.0, 0.005, 0.001, 0.025, 0.0025, 0.0025 / 20, 0.0025]
SHAPES = [(1001, 3), (1001, 3), (1001, 4), (1001, 1), (1001, 1, 3), (1001, 15, 3), (1001, 33)]


def _leaves(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g).cuda().requires_grad_(True) for s in SHAPES]


def _grads(seed, step):
    g = torch.Generator().manual_seed(seed * 100 + step)
    return [torch.randn(*s, generator=g).cuda() for s in SHAPES]


def test_flat_adam_matches_torch_fused_adam_and_oracle():
    from hds_b200.optim import FlatAdam

    ours = _leaves(0)
    ref = [p.detach().clone().requires_grad_(True) for p in ours]
    start = [p.detach().cpu().numpy().copy() for p in ours]
    opt = FlatAdam(ours, LRS, eps=1e-15)
    torch_opt = torch.optim.Adam([{"params": [p], "lr": lr} for p, lr in zip(ref, LRS)], eps=1e-15, fused=True)
    o_state = [(x, np.zeros_like(x), np.zeros_like(x)) for x in start]
    for step in range(1, 4):
        grads = _grads(0, step)
        opt.zero_grad()
        for p, gr in zip(ours, grads):
            p.grad.copy_(gr)
        opt.step()
        for p, gr in zip(ref, grads):
            p.grad = gr.clone()
        torch_opt.step()
        o_state = [oracle.adam(x, m, v, gr.cpu().numpy(), step, lr, 0.9, 0.999, 1e-15)
                   for (x, m, v), gr, lr in zip(o_state, grads, LRS)]
    for i, (p, r, (x, m, v)) in enumerate(zip(ours, ref, o_state)):
        got = p.detach().cpu().numpy()
        assert np.array_equal(got, x), f"group {i}: parameters differ from the oracle's Adam"
        n0 = sum(int(np.prod(s)) for s in SHAPES[:i])
        n1 = n0 + int(np.prod(SHAPES[i]))
        assert np.array_equal(opt.exp_avg[n0:n1].cpu().numpy(), m.reshape(-1)), f"group {i}: exp_avg differs"
        assert np.array_equal(opt.exp_avg_sq[n0:n1].cpu().numpy(), v.reshape(-1)), f"group {i}: exp_avg_sq differs"
        # torch's fused kernel rounds its bias corrections and update differently: parameters agree to
        # about 1e-6 of the three steps' movement (lr each).
        np.testing.assert_allclose(got, r.detach().cpu().numpy(), rtol=1e-6, atol=1e-5 * 3 * LRS[i],
                                   err_msg=f"group {i} vs torch.optim.Adam(fused=True)")
        # The leaf is still the caller's tensor, now a view of the flat buffer.
        assert p.data_ptr() == opt.flat[n0:n1].data_ptr()


def test_adam_step_unaligned_buffers_take_the_element_path():
    from hds_b200.optim import adam_step

    n = 4099
    rng = np.random.default_rng(3)
    arrays = [rng.standard_normal(n).astype(np.float32) for _ in range(2)]
    p0, g0 = arrays
    bufs = []
    for a in (p0, np.zeros(n, np.float32), np.zeros(n, np.float32), g0):
        big = torch.zeros(n + 1, device="cuda")
        big[1:] = torch.from_numpy(a).cuda()
        bufs.append(big[1:])
    ends, lrs = [1000, 1001, n], [0.01, 0.02, 0.03]
    adam_step(*bufs, ends, lrs, 1)
    want_p = p0.copy()
    for (a, b), lr in zip(zip([0] + ends[:-1], ends), lrs):
        want_p[a:b] = oracle.adam(p0[a:b], np.zeros(b - a, np.float32), np.zeros(b - a, np.float32), g0[a:b], 1, lr,
                                  0.9, 0.999, 1e-15)[0]
    assert np.array_equal(bufs[0].cpu().numpy(), want_p)


def test_sharded_flat_adam_on_one_rank_equals_flat_adam():
    """ShardedFlatAdam over a one-rank NCCL group (the reduce-scatter and all-gather are copies, the
    padded shard holds every parameter) steps exactly as FlatAdam: three steps, bit for bit.  The
    sharding across ranks is checked with gloo ranks on the CPU."""
    import os
    import socket

    import torch.distributed as dist

    from hds_b200.optim import FlatAdam, ShardedFlatAdam

    if dist.is_initialized():
        pytest.skip("a process group is already initialised in this process")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        a, b = _leaves(3), _leaves(3)
        flat = FlatAdam(a, LRS, eps=1e-15)
        sharded = ShardedFlatAdam(b, LRS, eps=1e-15)
        assert sharded.shard % 64 == 0 and sharded.shard >= flat.flat.numel()
        for step in range(1, 4):
            grads = _grads(3, step)
            flat.zero_grad()
            sharded.zero_grad()
            for p, q, gr in zip(a, b, grads):
                p.grad.add_(gr)
                q.grad.add_(gr)
            flat.step()
            sharded.step()
        torch.cuda.synchronize()
        for p, q in zip(a, b):
            assert torch.equal(p.detach(), q.detach())
    finally:
        dist.destroy_process_group()


def test_flat_adam_with_head_and_tail_reserves_steps_only_the_parameters():
    """FlatAdam(head=, tail=) keeps zero reserves before and after the parameters in the flat buffer
    and the bucket (the tile-row split renders fetched rows there): the parameters step exactly as
    without reserves, and the reserves are neither stepped nor touched."""
    from hds_b200.optim import FlatAdam

    a, b = _leaves(5), _leaves(5)
    plain = FlatAdam(a, LRS, eps=1e-15)
    head, tail = 24, 40
    reserved = FlatAdam(b, LRS, eps=1e-15, head=head, tail=tail)
    n = plain.n
    assert reserved.flat.numel() == head + n + tail and reserved.bucket.flat.numel() == head + n + tail
    assert b[0].data_ptr() == reserved.flat[head:].data_ptr()
    for step in range(1, 4):
        grads = _grads(5, step)
        plain.zero_grad()
        reserved.zero_grad()
        for p, q, gr in zip(a, b, grads):
            p.grad.add_(gr)
            q.grad.add_(gr)
        # Whatever lands in the reserves (rows rendered beside the parameters) is not stepped.
        reserved.bucket.flat[:head] = 1.0
        reserved.bucket.flat[head + n:] = 1.0
        reserved.flat[:head] = 7.0
        plain.step()
        reserved.step()
    torch.cuda.synchronize()
    for p, q in zip(a, b):
        assert torch.equal(p.detach(), q.detach())
    assert torch.all(reserved.flat[:head] == 7.0) and torch.all(reserved.flat[head + n:] == 0.0)
