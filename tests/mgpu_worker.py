"""Worker for tests/test_multi_gpu.py, run under torch.distributed.run (one rank per GPU).

Modes (argv[1]):
  parity   sharded run() with the in-kernel peer exchange and with NCCL, against
           the single-GPU runtime on rank 0: prints "PARITY <case> <bool>".
  timeout  rank 1 stays alive but does not launch; rank 0's kernel must end
           with status code 6 (its cross-GPU barrier gave up): prints "STATUS <code>".
  checkpoint  a sharded run is captured into one payload and restored into a
           fresh sharded run and into a single-GPU runtime; both continue bit
           for bit like the original: prints "CHECKPOINT <case> <bool>".
  pels     row-sharded PELS with the peer and the NCCL delta exchange: 4 ticks
           against the single-GPU PELS runtime, then a CUDA-graph run; theta = 0
           against the matrix tick and the current against W @ emitted; then
           B = 1 hybrid ticks over the peer exchange: prints
           "PELS <exchange>-<theta> <bool> ..." and "PELS hybrid-peer <bool> ...".
  pels_timeout  rank 1 stays alive but does not launch; rank 0's scatter must
           end its bounded cross-GPU wait with status code 6: prints "STATUS <code>".
  stream   sharded stream() (per-tick drives of the rank's rows, every tick's
           rows copied out) with the peer exchange (rollout launches) and with
           NCCL, interleaved with run(), against single-GPU steps with the same
           drives: prints "STREAM <exchange> <bool>".
"""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from neurosim_gpu_b200 import (DendriticDynamics, Dynamics,  # noqa: E402
                               NativeDendriticMatrixRuntime, random_topology)
from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime, broadcast_graph  # noqa: E402


def model(n, device):
    soma = Dynamics(torch.linspace(0.5, 0.9, n, device=device), torch.full((n,), 0.8, device=device))
    return DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                 tau_adaptation=25.0, coupling=0.5,
                                                 adaptation_strength=0.2)


def parity(device, rank):
    for n, m, precision, exchange in ((20011, 500000, "fp32", "peer"),
                                      (20011, 500000, "nvfp4", "peer"),
                                      (20011, 500000, "fp32", "nccl")):
        graph = broadcast_graph(n, m, seed=4, device=device)
        dyn = model(n, device)
        init = torch.rand(1, n, generator=torch.Generator().manual_seed(3)).to(device)
        rt = ShardedDendriticMatrixRuntime(graph, dyn, init, precision=precision, exchange=exchange)
        with torch.inference_mode():
            rt.run(9, 0.2, dendritic_drive=0.1, graph_ticks=4)
            rt.step(0.2, dendritic_drive=0.1)
            rt.run(7, 0.25, dendritic_drive=0.1, graph_ticks=4)
        torch.cuda.synchronize()
        state = rt.state.clone()
        dendrite = rt.gather("dendritic_state")
        rt.check_status()
        rt.release_graphs()
        rt.close()
        if rank == 0:
            topo = random_topology(n, m, device="cpu", seed=4, build_device=device)
            single = NativeDendriticMatrixRuntime(topo, dyn, init.clone(), precision=precision,
                                                  kernel="tiled")
            with torch.inference_mode():
                for k in range(17):
                    single.step(0.2 if k < 10 else 0.25, dendritic_drive=0.1)
            torch.cuda.synchronize()
            ok = torch.equal(state, single.state) and torch.equal(dendrite, single.dendritic_state)
            ds = float((state - single.state).abs().max())
            dd = float((dendrite - single.dendritic_state).abs().max())
            print(f"PARITY {precision}-{exchange} {ok} state_diff={ds:.3g} dendrite_diff={dd:.3g}",
                  flush=True)
        dist.barrier()


def timeout(device, rank):
    n, m = 20011, 500000
    graph = broadcast_graph(n, m, seed=4, device=device)
    rt = ShardedDendriticMatrixRuntime(graph, model(n, device), torch.zeros(1, n, device=device),
                                       exchange="peer")
    if rank == 0:
        with torch.inference_mode():
            rt.run(1, 0.2, dendritic_drive=0.1)  # rank 1 never arrives: bounded wait, code 6
        torch.cuda.synchronize()
        print(f"STATUS {int(rt.status.item())}", flush=True)
    else:
        # The host side of run() (its pre-launch barrier) without the launch.
        torch.cuda.synchronize()
        dist.barrier()
    dist.barrier()  # rank 1 waits here, alive, with nothing in flight
    rt.close()


def checkpoint(device, rank):
    from neurosim_gpu_b200.checkpoint import (capture_sharded_runtime, restore_runtime,
                                              restore_sharded_runtime)
    n, m = 20011, 500000
    graph = broadcast_graph(n, m, seed=4, device=device)
    dyn = model(n, device)
    init = torch.rand(1, n, generator=torch.Generator().manual_seed(3)).to(device)
    rt = ShardedDendriticMatrixRuntime(graph, dyn, init)
    with torch.inference_mode():
        rt.run(6, 0.2, dendritic_drive=0.1)
    topology = random_topology(n, m, device="cpu", seed=4) if rank == 0 else None
    payload = capture_sharded_runtime(rt, topology)
    with torch.inference_mode():
        rt.run(5, 0.2, dendritic_drive=0.1)
    want = rt.state.clone()
    box = [payload]
    dist.broadcast_object_list(box, src=0)
    again = ShardedDendriticMatrixRuntime(graph, dyn, torch.zeros(1, n, device=device))
    restore_sharded_runtime(again, box[0])
    with torch.inference_mode():
        again.run(5, 0.2, dendritic_drive=0.1)
    same_sharded = torch.equal(again.state, want)
    for runtime in (rt, again):
        runtime.release_graphs()
        runtime.close()
    if rank == 0:
        print(f"CHECKPOINT sharded {same_sharded}", flush=True)
        single = NativeDendriticMatrixRuntime(topology.to(device), dyn,
                                              torch.zeros(1, n, device=device), kernel="tiled")
        restore_runtime(single, payload)
        with torch.inference_mode():
            single.run(5, 0.2, dendritic_drive=0.1)
        print(f"CHECKPOINT single {torch.equal(single.state, want)}", flush=True)
    dist.barrier()


def pels(device, rank):
    from neurosim_gpu_b200 import NativeDendriticPELSRuntime
    from neurosim_gpu_b200.native import load_native_extension
    from neurosim_gpu_b200.sharded_pels import ShardedDendriticPELSRuntime
    n, m, batch = 20011, 500000, 2
    graph = broadcast_graph(n, m, seed=4, device=device)
    dyn = model(n, device)
    init = torch.rand(batch, n, generator=torch.Generator().manual_seed(3)).to(device)
    ext = load_native_extension()
    names = ("state", "dendritic_state", "adaptation_state", "emitted_state",
             "persistent_current")
    for exchange in ("peer", "nccl"):
        for theta in (0.02, 0.0):
            rt = ShardedDendriticPELSRuntime(graph, dyn, init, theta=theta, exchange=exchange)
            with torch.inference_mode():
                for _ in range(4):
                    rt.step(0.2, dendritic_drive=0.1)
                early = {name: rt.gather(name) for name in names}
                rt.run(16, 0.2, dendritic_drive=0.1, graph_ticks=8)
                rt.step(0.2, dendritic_drive=0.1)
                late = {name: rt.gather(name) for name in names}
            torch.cuda.synchronize()
            status = int(rt.status.item())
            path = rt.exchange
            rt.release_graphs()
            rt.close()
            if rank == 0:
                topo = random_topology(n, m, device="cpu", seed=4, build_device=device)
                single = NativeDendriticPELSRuntime(topo, dyn, init.clone(), theta=theta)
                with torch.inference_mode():
                    for _ in range(4):
                        single.step(0.2, dendritic_drive=0.1)
                diff = max(float((early[k] - getattr(single, k)).abs().max()) for k in names)
                product = ext.csr_propagate(topo.in_rowptr, topo.in_col, topo.in_weight,
                                            late["emitted_state"].contiguous())
                drift = float((late["persistent_current"] - product).abs().max())
                ok = path == exchange and status == 0 and diff <= 2e-6 and drift <= 2e-5
                extra = ""
                if theta == 0.0:
                    matrix = NativeDendriticMatrixRuntime(topo, dyn, init.clone(), kernel="csr")
                    with torch.inference_mode():
                        for _ in range(21):
                            matrix.step(0.2, dendritic_drive=0.1)
                    gap = float((late["state"] - matrix.state).abs().max())
                    ok = ok and gap <= 8e-6
                    extra = f" matrix_gap={gap:.3g}"
                print(f"PELS {exchange}-{theta} {ok} diff={diff:.3g} drift={drift:.3g} "
                      f"status={status}{extra}", flush=True)
            dist.barrier()
    # B = 1 hybrid ticks over the peer exchange: the activity of all ranks picks
    # the scatter or the tiled propagate (gate 5 % of M: both occur).
    init1 = init[:1].contiguous()
    rt = ShardedDendriticPELSRuntime(graph, dyn, init1, theta=0.02, exchange="peer",
                                     propagation="hybrid", hybrid_gate=0.05)
    with torch.inference_mode():
        for t in range(4):
            rt.step(0.2 + 0.1 * t, dendritic_drive=0.1)
        early = {name: rt.gather(name) for name in names}
        rt.run(16, 0.3, dendritic_drive=0.1, graph_ticks=8)
        late = {name: rt.gather(name) for name in names}
    torch.cuda.synchronize()
    status = int(rt.status.item())
    mode = rt.propagation
    rt.release_graphs()
    rt.close()
    if rank == 0:
        topo = random_topology(n, m, device="cpu", seed=4, build_device=device)
        single = NativeDendriticPELSRuntime(topo, dyn, init1.clone(), theta=0.02,
                                            propagation="event")
        with torch.inference_mode():
            for t in range(4):
                single.step(0.2 + 0.1 * t, dendritic_drive=0.1)
        diff = max(float((early[k] - getattr(single, k)).abs().max()) for k in names)
        product = ext.csr_propagate(topo.in_rowptr, topo.in_col, topo.in_weight,
                                    late["emitted_state"].contiguous())
        drift = float((late["persistent_current"] - product).abs().max())
        ok = mode == "hybrid" and status == 0 and diff <= 2e-6 and drift <= 2e-5
        print(f"PELS hybrid-peer {ok} diff={diff:.3g} drift={drift:.3g} status={status}",
              flush=True)
    dist.barrier()


def pels_timeout(device, rank):
    from neurosim_gpu_b200.sharded_pels import ShardedDendriticPELSRuntime
    n, m = 20011, 500000
    graph = broadcast_graph(n, m, seed=4, device=device)
    rt = ShardedDendriticPELSRuntime(graph, model(n, device), torch.zeros(1, n, device=device),
                                     theta=0.0, exchange="peer")
    if rank == 0:
        with torch.inference_mode():
            rt.step(0.2, dendritic_drive=0.1)  # rank 1 never signals: bounded wait, code 6
        torch.cuda.synchronize()
        print(f"STATUS {int(rt.status.item())}", flush=True)
    dist.barrier()  # rank 1 waits here, alive, with nothing in flight
    rt.close()


def stream(device, rank):
    n, m = 20011, 500000
    graph = broadcast_graph(n, m, seed=4, device=device)
    dyn = model(n, device)
    init = torch.rand(1, n, generator=torch.Generator().manual_seed(3)).to(device)
    drives = torch.rand(48, 1, n, generator=torch.Generator().manual_seed(8)) * 0.4
    topo = random_topology(n, m, device="cpu", seed=4, build_device=device)
    single = NativeDendriticMatrixRuntime(topo, dyn, init.clone(), kernel="tiled")
    want = []
    with torch.inference_mode():
        for t in range(45):
            want.append(single.step(drives[t].to(device), dendritic_drive=0.1).clone())
        for _ in range(5):
            single.step(0.2, dendritic_drive=0.1)
        for t in range(45, 48):
            want.append(single.step(drives[t].to(device), dendritic_drive=0.1).clone())
    torch.cuda.synchronize()
    for exchange in ("peer", "nccl"):
        rt = ShardedDendriticMatrixRuntime(graph, dyn, init, exchange=exchange)
        lo, hi = rt.shard.lo, rt.shard.hi
        mine = drives[:, :, lo:hi].contiguous().pin_memory()
        with torch.inference_mode():
            first = rt.stream(mine[:45], dendritic_drive=0.1)  # launches of 4, 8, 21, 8, 4 ticks
            rt.run(5, 0.2, dendritic_drive=0.1, graph_ticks=4)
            second = rt.stream(mine[45:, 0], dendritic_drive=0.1)  # [T, rows] drives
        torch.cuda.synchronize()
        got = torch.cat([first, second])
        ok = rt.exchange == exchange and all(
            torch.equal(got[t].to(device), want[t][:, lo:hi]) for t in range(48))
        ok = ok and torch.equal(rt.state, single.state) and int(rt.status.item()) == 0
        flag = torch.tensor([int(ok)], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        rt.release_graphs()
        rt.close()
        if rank == 0:
            print(f"STREAM {exchange} {bool(flag.item())}", flush=True)
        dist.barrier()


def main():
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        {"parity": parity, "timeout": timeout, "checkpoint": checkpoint, "pels": pels,
         "pels_timeout": pels_timeout, "stream": stream}[sys.argv[1]](
            device, dist.get_rank())
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
