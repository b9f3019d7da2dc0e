"""The allocation-free PELS entry point (nsb_dendritic_event_noalloc).

It exists for hosts that cannot give the library scratch memory: an
application whose device memory is all reserved up front by its own pool and
that may not allocate inside its simulation loop, or a foreign-language host
(cgo, JNI, ...) that holds plain device pointers but no CUDA allocator.  This
file is named to be collected last, so a run that stops at its first failure
has run every other test first; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

from neurosim_gpu_b200 import load_native_extension, random_topology
from neurosim_gpu_b200.dynamics import DendriticDynamics, Dynamics

pytestmark = pytest.mark.gpu


def _case(n=3000, batch=4, edges=60000):
    graph = random_topology(n, edges, device="cpu", seed=11).to("cuda")
    soma = Dynamics(torch.linspace(0.5, 0.9, n, device="cuda"),
                    torch.full((n,), 0.8, device="cuda"))
    model = DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                  tau_adaptation=25.0, coupling=0.5,
                                                  adaptation_strength=0.2)
    state = torch.rand(batch, n, generator=torch.Generator().manual_seed(3)).cuda()
    return graph, model, state


def test_noalloc_event_matches_workspace_entry_point_on_two_calls():
    ext = load_native_extension()
    graph, model, state = _case()
    params = model.parameters()
    theta = torch.full((graph.n_neurons,), 0.01, device="cuda")
    dendrite = torch.zeros_like(state)
    adaptation = torch.zeros_like(state)
    emitted = torch.zeros_like(state)
    current = ext.csr_propagate(graph.in_rowptr, graph.in_col, graph.in_weight, emitted)
    inputs = (state, dendrite, adaptation, emitted)
    for _ in range(2):  # the second call finds the first call's leftovers in the scratch
        current_a, current_b = current.clone(), current.clone()
        ra = ext.dendritic_event(*inputs[:3], params, current_a, inputs[3], theta,
                                 graph.out_rowptr, graph.dst, None, graph.weight, None, 0.3,
                                 None, 0.1)
        rb = ext.dendritic_event_noalloc(*inputs[:3], params, current_b, inputs[3], theta,
                                         graph.out_rowptr, graph.dst, None, graph.weight, None,
                                         0.3, None, 0.1)
        # The update and emit rule are deterministic: identical states.
        for got, want in zip(rb, ra):
            torch.testing.assert_close(got, want, atol=0, rtol=0)
        # The scatter adds with float atomics in no fixed order: the PELS tolerance.
        torch.testing.assert_close(current_b, current_a, atol=1e-6, rtol=0)
        assert int((rb[3] != inputs[3]).sum()) > 0  # sources did emit
        inputs, current = tuple(ra), current_a


def test_noalloc_event_rejects_sizes_beyond_its_scratch():
    ext = load_native_extension()
    n = 300_000
    graph = random_topology(n, 1000, device="cpu", seed=2).to("cuda")
    soma = Dynamics(torch.full((n,), 0.7, device="cuda"), torch.full((n,), 0.8, device="cuda"))
    model = DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                  tau_adaptation=25.0)
    state = torch.zeros(4, n, device="cuda")  # 1.2M pairs > 2^20
    with pytest.raises(RuntimeError, match="exceeds its fixed scratch"):
        ext.dendritic_event_noalloc(state, state, state, model.parameters(), state.clone(), state,
                                    torch.zeros(n, device="cuda"), graph.out_rowptr, graph.dst,
                                    None, graph.weight, None, 0.0, None, 0.0)


def test_noalloc_event_allocates_no_device_memory():
    """The property the entry point exists for: with the caller's outputs given,
    repeated calls leave the device's free memory and torch's allocator alone."""
    ext = load_native_extension()
    graph, model, state = _case()
    params = model.parameters()
    theta = torch.full((graph.n_neurons,), 0.01, device="cuda")
    current = torch.zeros_like(state)
    states = [[state.clone(), torch.zeros_like(state), torch.zeros_like(state),
               torch.zeros_like(state)] for _ in range(2)]

    def call(k):
        s, d, a, e = states[k]
        ext.dendritic_event_noalloc(s, d, a, params, current, e, theta, graph.out_rowptr,
                                    graph.dst, None, graph.weight, None, 0.3, None, 0.1,
                                    out=states[1 - k])

    call(0)  # the first call in this context looks up the scratch address
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    allocated_before = torch.cuda.memory_allocated()
    reserved_before = torch.cuda.memory_reserved()
    for k in (1, 0, 1, 0):
        call(k)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert torch.cuda.memory_allocated() == allocated_before
    assert torch.cuda.memory_reserved() == reserved_before
    assert bool(torch.isfinite(states[1][0]).all())
    assert int((states[1][3] != 0).sum()) > 0  # sources did emit
