"""Host-side sequence split and KV-head sharding over gloo ranks (no GPU).

Two CPU processes share a seeded paged problem; each computes the partial
attention state of its page-aligned token range with the CPU oracle, packs it
as SeqSplitAttention does ([O rows*D | LSE rows] fp32), the packed buffers
are all-gathered over gloo and merged (oracle merge) on every rank; the result
must equal the oracle over the whole sequence.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle import merge as oracle_merge
from helm_b200.runtime.seq_parallel import SeqSplitAttention, head_range, split_ranges


def test_split_ranges_are_page_aligned_and_cover():
    for total, P, world in [(131072, 16, 8), (1000, 16, 3), (5, 16, 4), (0, 16, 2), (640, 64, 2)]:
        r = split_ranges(total, P, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == total
        for (a, b), (c, d) in zip(r, r[1:]):
            assert b == c and a <= b
            assert a % P == 0 and (b % P == 0 or b == total)


def test_head_range():
    assert head_range(8, 40, 3, 8) == ((3, 4), (15, 20))
    assert head_range(40, 40, 1, 8) == ((5, 10), (5, 10))
    with pytest.raises(ValueError):
        head_range(8, 32, 0, 3)


def _problem(seed=0, B=2, Hq=8, Hkv=2, D=64, P=16, lens=(300, 77)):
    g = torch.Generator().manual_seed(seed)
    maxp = max(-(-L // P) for L in lens)
    slots = B * maxp + 3
    perm = torch.randperm(slots, generator=g)
    pt = perm[:B * maxp].view(B, maxp).to(torch.int32).numpy()
    pool = torch.randn(slots, 2, Hkv, P, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    bits = pool.view(torch.int16).numpy().view(np.uint16)
    return q.float().numpy(), bits, pt, np.array(lens), dict(B=B, Hq=Hq, Hkv=Hkv, D=D, P=P)


def _range_lists(pt, lens, P, rng):
    """Page lists of one token range (ragged form, as the oracle takes them)."""
    B = pt.shape[0]
    a, b = rng
    maxp = pt.shape[1]
    sub = np.zeros((B, maxp), np.int32)
    used = np.zeros((B, maxp), np.int32)
    nump = np.zeros(B, np.int32)
    for i in range(B):
        lo, hi = min(a, lens[i]), min(b, lens[i])
        k = 0
        for page in range(lo // P, -(-hi // P) if hi > 0 else 0):
            s, e = max(lo, page * P), min(hi, (page + 1) * P)
            if e <= s:
                continue
            sub[i, k] = pt[i, page]
            used[i, k] = e - s
            k += 1
        nump[i] = k
    return sub, nump, used


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, bits, pt, lens, m = _problem()
        rows, D = m["B"] * m["Hq"], m["D"]
        rng = split_ranges(int(lens.max()), m["P"], world)[rank]
        sub, nump, used = _range_lists(pt, lens, m["P"], rng)
        o, lse = oracle.paged_attention(q, bits, oracle.DT_BF16, sub, nump, used,
                                        num_kv_heads=m["Hkv"], page_size=m["P"], scale=D ** -0.5)
        part = torch.from_numpy(np.concatenate([o.reshape(-1), lse.reshape(-1)]).astype(np.float32))

        def merge_fn(o_parts, lse_parts, dtype):
            mo, ml = oracle_merge.merge_states(o_parts.numpy(), lse_parts.numpy())
            return torch.from_numpy(mo), torch.from_numpy(ml)

        sp = SeqSplitAttention(merge_fn=merge_fn)
        gathered = sp.exchange(part)
        out, lse_m = sp.merge(gathered, rows, D, torch.float32)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(out_dir, f"lse{rank}.npy"), lse_m.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_two_ranks_sequence_split_equals_full(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    q, bits, pt, lens, m = _problem()
    nump, used = oracle.dense_page_lists(lens, m["P"], pt.shape[1])
    full, full_lse = oracle.paged_attention(q, bits, oracle.DT_BF16, pt, nump, used,
                                            num_kv_heads=m["Hkv"], page_size=m["P"],
                                            scale=m["D"] ** -0.5)
    for r in range(world):
        out = np.load(tmp_path / f"out{r}.npy")
        lse = np.load(tmp_path / f"lse{r}.npy")
        np.testing.assert_allclose(out, full.reshape(out.shape), rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(lse, full_lse.reshape(-1), rtol=1e-6, atol=1e-5)


def _leaving_worker(rank, world, port, out_dir):
    """Both ranks finish one exchange; rank 1 then leaves between steps
    (nothing in flight); rank 0's next exchange must end with an error within
    the process group's timeout instead of waiting for good."""
    import time
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    sp = SeqSplitAttention()
    part = torch.full((6,), float(rank))
    first = sp.exchange(part)
    if rank == 1:
        os._exit(0)  # departs without a further collective
    t0 = time.time()
    try:
        sp.exchange(part)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - the kind of error is backend-specific
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome}\n{time.time() - t0:.2f}\n{first.tolist()}\n")
    os._exit(0)


def test_departed_rank_ends_the_next_exchange_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    outcome, elapsed, first = (tmp_path / "rank0.txt").read_text().splitlines()
    assert outcome.startswith("error"), outcome
    assert float(elapsed) < 60
    assert first == str([[0.0] * 6, [1.0] * 6])


def test_sequence_split_token_ownership():
    """Model-level sequence split (runtime/seq_decode.py): for every position,
    exactly one rank writes the token's K/V row (the one whose range holds it;
    the last rank past the context), at its own next row; over all ranks a
    query attends each of the pos + 1 tokens once."""
    from helm_b200.runtime.seq_decode import token_rows
    for T, P, world, extra in [(100, 16, 2, 20), (131072, 16, 8, 5), (40, 16, 4, 3), (64, 64, 2, 70)]:
        ranges = split_ranges(T, P, world)
        L, B = 2, 3
        tabs, caps = [], []
        for r, (a, b) in enumerate(ranges):
            cap = (b - a) + (extra if r == world - 1 else 0)
            maxp = max(1, -(-cap // P))
            base = torch.arange(L * B, dtype=torch.int32).view(L, B, 1) * maxp
            tabs.append(base + torch.arange(maxp, dtype=torch.int32))
            caps.append(cap)
        for p in list(range(0, min(T + extra, 300))) + list(range(T, T + extra)):
            pos = torch.full((B,), p, dtype=torch.int32)
            owners, total = [], torch.zeros(B, dtype=torch.int64)
            for r, rng in enumerate(ranges):
                rows, lens = token_rows(pos, rng, r == world - 1, caps[r], tabs[r], P)
                total += lens.long()
                if bool((rows >= 0).all()):
                    owners.append(r)
                    li = p - rng[0]
                    want = tabs[r][:, :, li // P].long() * P + li % P
                    assert torch.equal(rows, want)
                else:
                    assert bool((rows == -1).all())
            assert len(owners) == 1, (T, world, p, owners)
            a, b = ranges[owners[0]]
            assert a <= p and (p < b or owners[0] == world - 1)
            assert bool((total == p + 1).all()), (T, world, p, total)
