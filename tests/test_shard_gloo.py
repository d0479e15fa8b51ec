"""The multi-GPU path's host logic on CPU, with two gloo ranks: each rank
computes its row slice of a projection (the reference's algorithm, via the
oracle) from the splits bench.py uses, the slices are all-gathered, and the
result equals the unsharded product bit for bit - a row does not depend on the
split (lab_native.c:550-552). The sharded chain's tiled split must also start
every slice on a 32-row tile and cover every row exactly once. The head path
(decoder layers whole on every rank, only the lm_head's rows split) must give
the unsharded stack's logits bit for bit, gathered by bench.py's own helper
(three ranks split the 1000 vocabulary rows unevenly)."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

CASES = [("q8", 4096, 256), ("q8", 1000, 128), ("q4", 2048, 512), ("q8", 151936 // 64, 64)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    from oracle import oracle as orc
    o = orc.Oracle()
    results = []
    for tiled in (False, True):
        for fmt, rows, cols in CASES:
            rng = np.random.default_rng(rows + cols)
            qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
            x = orc.activations(rng, 1, cols)
            r0, r1 = bench.row_split(rows, rank, world, tiled)
            wb = cols // 2 if fmt == "q4" else cols
            y, _, _ = o.gemm(fmt, qs[r0 * wb:r1 * wb], sc[r0 * (cols // 32):r1 * (cols // 32)], x,
                             r1 - r0, cols, 1, 1)
            parts = [None] * world
            dist.all_gather_object(parts, (r0, r1, y))
            if rank == 0:
                want, _, _ = o.gemm(fmt, qs, sc, x, rows, cols, 1, 1)
                got = np.concatenate([p[2] for p in sorted(parts, key=lambda p: p[0])])
                spans = sorted((p[0], p[1]) for p in parts)
                results.append((tiled, fmt, rows, cols, spans,
                                bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))))
    # The head path: layers whole on every rank, the lm_head's rows split;
    # the gathered logits equal one rank's run of the whole stack.
    rng = np.random.default_rng(7)
    hidden, ffn, vocab = 64, 96, 1000
    mats = [("q8", "o", hidden, hidden), ("q4", "up", ffn, hidden), ("q8", "down", hidden, ffn),
            ("q8", "lm_head", vocab, hidden)]
    weights = [orc.q4_weights(rng, r, c) if f == "q4" else orc.q8_weights(rng, r, c) for f, _, r, c in mats]
    x0 = orc.activations(rng, 1, hidden)

    def run(shard):
        x = x0
        for (fmt, name, rows, cols), (qs, sc) in zip(mats, weights):
            r0, r1 = bench.shard_rows(name, rows, rank, world, "head") if shard else (0, rows)
            wb = cols // 2 if fmt == "q4" else cols
            y, _, _ = o.gemm(fmt, qs[r0 * wb:r1 * wb], sc[r0 * (cols // 32):r1 * (cols // 32)],
                             x.reshape(1, cols), r1 - r0, cols, 1, 1)
            x = y.reshape(-1)
        return r0, r1, x

    r0, r1, part = run(True)
    # The logits gathered by bench.py's own helper (in place, any split).
    logits = torch.full((vocab,), float("nan"))
    logits[r0:r1] = torch.from_numpy(part)
    bench.make_gather(dist, rank, world)(logits)
    parts = [None] * world
    dist.all_gather_object(parts, (r0, r1, part))
    if rank == 0:
        want = run(False)[2]
        got = np.concatenate([p[2] for p in sorted(parts, key=lambda p: p[0])])
        spans = sorted((p[0], p[1]) for p in parts)
        same = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)) and
                    np.array_equal(logits.numpy().view(np.uint32), want.view(np.uint32)))
        results.append(("head", "stack", vocab, hidden, spans, same))
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        out.put(results)


@pytest.mark.parametrize("world", [2, 3])
def test_row_shards_reassemble_bit_exactly(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    results = q.get()
    assert len(results) == 2 * len(CASES) + 1
    for tiled, fmt, rows, cols, spans, same in results:
        assert same, (tiled, fmt, rows, cols)
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))  # contiguous, no overlap
        if tiled is True:
            assert all(s[0] % 32 == 0 for s in spans)
