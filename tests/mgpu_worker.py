"""Worker for tests/test_multi_gpu.py, run under torch.distributed.run (one rank per GPU).

Modes (argv[1]):
  parity   sharded run() with the in-kernel peer exchange and with NCCL, against
           the single-GPU runtime on rank 0: prints "PARITY <case> <bool>".
  timeout  rank 1 stays alive but does not launch; rank 0's kernel must end
           with status code 6 (its cross-GPU barrier gave up): prints "STATUS <code>".
  checkpoint  a sharded run is captured into one payload and restored into a
           fresh sharded run and into a single-GPU runtime; both continue bit
           for bit like the original: prints "CHECKPOINT <case> <bool>".
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


def main():
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        {"parity": parity, "timeout": timeout, "checkpoint": checkpoint}[sys.argv[1]](
            device, dist.get_rank())
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
