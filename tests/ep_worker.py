"""Child-process bodies for the expert-parallel tests (one process per rank).

Each rank builds its expert shard and its rank workspace, exchanges the CUDA
IPC handles of the exported buffers over a gloo group on 127.0.0.1, runs the
expert-parallel forward of its own tokens and compares it with the
single-GPU forward of the same tokens on the full expert set."""
import os
import sys

import numpy as np


def _setup(rank, world, port, use_gpu, device=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    if use_gpu:
        import torch
        torch.cuda.set_device(rank if device is None else device)
    return dist


def exchange_worker(rank, world, port, queue):
    """Host plumbing only: all-gather of per-rank handle bytes."""
    try:
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        dist = _setup(rank, world, port, use_gpu=False)
        got = pkg.exchange_handles(bytes([rank + 1]) * pkg.EP_HANDLE_BYTES)
        queue.put((rank, [g[0] for g in got], len(got[0])))
        dist.destroy_process_group()
    except Exception as ex:  # reported to the parent
        queue.put((rank, "error", repr(ex)))


def forward_worker(rank, world, port, tokens, routing, queue):
    try:
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import torch
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        dist = _setup(rank, world, port, use_gpu=True)
        dev = torch.device("cuda", rank)
        desc = pkg.make_desc(max_tokens=tokens, device=rank)
        rng = np.random.default_rng(100 + rank)
        x = torch.from_numpy(rng.standard_normal((tokens, 2048)).astype(np.float32)).to(dev)
        if routing == "zipf":
            perm = np.random.default_rng(7).permutation(512)   # same skew on every rank
            g = -np.log(-np.log(rng.random((tokens, 512))))
            lg = (-1.1 * np.log1p(perm.astype(np.float64))[None, :] + g).astype(np.float32)
        else:
            lg = rng.standard_normal((tokens, 512)).astype(np.float32)
        logits = torch.from_numpy(lg).to(dev)
        gate = torch.from_numpy(np.random.default_rng(5).standard_normal(2048).astype(np.float32) * 0.05)
        # single-GPU result on the full expert set
        full = pkg.MoeWeights(desc)
        full.synthesize(11, 3)
        full.upload_shared_gate(gate.numpy())
        layer = pkg.MoeLayer(desc)
        ref = torch.zeros(tokens, 2048, device=dev)
        layer.forward(full, x, logits, ref)
        # expert-parallel result
        shard = pkg.EpWeights(desc, rank, world)
        shard.synthesize(11, 3)
        shard.upload_shared_gate(gate.numpy())
        ep = pkg.EpLayer(desc, rank, world)
        ep.connect(pkg.exchange_handles)
        outs = []
        for _ in range(2):   # two forwards: epochs advance, buffers are reused
            out = torch.zeros(tokens, 2048, device=dev)
            ep.forward(shard, x, logits, out)
            outs.append(out)
        torch.cuda.synchronize()
        flags = ep.read_flags() | layer.read_flags()
        r = ref.cpu().numpy()
        rms = float(np.sqrt(np.mean(r.astype(np.float64) ** 2)))
        errs = [float(np.abs(o.cpu().numpy() - r).max()) for o in outs]
        dist.barrier()
        ep.close()
        dist.barrier()
        queue.put((rank, flags, errs, rms))
        dist.destroy_process_group()
    except Exception as ex:
        queue.put((rank, "error", repr(ex), 0.0))


def silent_peer_worker(rank, world, port, queue):
    """Failure detection without a fault: both ranks live on GPU 0 and open each
    other's buffers, but rank 1 never runs a forward.  Rank 0's bounded waits
    (received slots, peers' "done") run out on flags nothing sets; the forward
    must return with MOE_FLAG_TIMEOUT in the rank's flags and the context must
    stay usable (a single-GPU forward afterwards is clean).  Rank 1 keeps its
    buffers alive until rank 0 is done; no two kernels wait on one another."""
    try:
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import time
        import torch
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        dist = _setup(rank, world, port, use_gpu=True, device=0)
        desc = pkg.make_desc(max_tokens=8, device=0)
        ep = pkg.EpLayer(desc, rank, world)
        ep.connect(pkg.exchange_handles)
        result = (rank, 0, 0.0, 0)
        if rank == 0:
            shard = pkg.EpWeights(desc, rank, world)
            shard.synthesize(5, 0)
            rng = np.random.default_rng(0)
            x = torch.from_numpy(rng.standard_normal((8, 2048)).astype(np.float32)).cuda()
            logits = torch.from_numpy(rng.standard_normal((8, 512)).astype(np.float32)).cuda()
            out = torch.zeros(8, 2048, device="cuda")
            t0 = time.time()
            ep.forward(shard, x, logits, out)
            flags = ep.read_flags()            # synchronises: the bounded waits have given up
            waited = time.time() - t0
            full = pkg.MoeWeights(desc)
            full.synthesize(5, 0)
            layer = pkg.MoeLayer(desc)
            ref = torch.zeros(8, 2048, device="cuda")
            layer.forward(full, x, logits, ref)
            torch.cuda.synchronize()
            result = (rank, flags, waited, layer.read_flags())
            ep.close()                          # the importer unmaps first
        dist.barrier()                          # rank 1 frees its buffers only after that
        if rank != 0:
            ep.close()
        dist.barrier()
        queue.put(result)
        dist.destroy_process_group()
    except Exception as ex:
        queue.put((rank, "error", repr(ex), 0))
