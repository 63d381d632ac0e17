"""Device-managed mode of an expert cache: its bookkeeping lives in HBM.

``GpuExpertCache`` normally keeps its slot bookkeeping on the host (the
native manager) and learns which experts a layer needs by reading the
router's result back, which puts a device-to-host synchronisation and a
host round trip in every layer that misses.  In device-managed mode the
same bookkeeping runs on the GPU (``csrc/expert_directory.cu``): a one-CTA
planning kernel takes the lease / eviction / fill decisions the host path
would take for the dispatch's experts, a fill kernel copies the missing
experts from page-locked host memory into their slots (SM loads over PCIe),
and the grouped SwiGLU runs once per wave.  Nothing in a layer waits for the
host, so a whole verify pass with misses can be captured in one CUDA graph.

The decisions are the host path's (``Qwen3OffloadedExperts._forward_waves``
over ``GpuExpertCache.acquire`` / ``release``): after ``leave`` (or any
read of the cache's statistics or snapshot) the host manager holds exactly
the slots, generations, LRU order and counters the host path would have
produced.  Device-managed mode has no leases or observer records per access
and runs canonical reductions only.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _native as N


class DeviceExpertDirectory:
    """The HBM copy of one cache's bookkeeping plus its per-wave buffers."""

    def __init__(self, cache) -> None:
        dev = cache.device
        E, S = len(cache._keys), cache.slot_count
        self.E, self.S = E, S
        self.waves = -(-E // S)  # ceil(E / S): a wave holds up to S experts
        i32 = dict(dtype=torch.int32, device=dev)
        i64 = dict(dtype=torch.int64, device=dev)
        self.slot_expert = torch.empty(S, **i32)
        self.slot_gen = torch.empty(S, **i32)
        self.slot_stamp = torch.empty(S, **i64)
        self.expert_slot = torch.empty(E, **i32)
        self.clock = torch.empty(1, **i64)
        self.counters = torch.empty(4, **i64)
        self.status = torch.zeros(1, **i32)
        W = self.waves
        self.wave_table = torch.empty(W, E, **i32)
        self.wave_active = torch.empty(W, E, **i32)
        self.wave_count = torch.empty(W, **i32)
        self.fill_expert = torch.empty(W, S, **i32)
        self.fill_slot = torch.empty(W, S, **i32)
        self.fill_count = torch.empty(W, **i32)
        addrs = []
        for key in cache._keys:
            src = cache._sources[key]
            out = ctypes.c_uint64()
            N.check(N.lib.sf_host_device_address(ctypes.c_void_p(src.data_ptr()), ctypes.byref(out)),
                    "device-managed expert cache")
            addrs.append(out.value)
        self.src_addr = torch.tensor(addrs, dtype=torch.int64).to(dev)
        first = cache._sources[cache._keys[0]]
        self.expert_bytes = first.numel() * first.element_size()
        self.fill_grid = 2 * torch.cuda.get_device_properties(dev).multi_processor_count

    # ------------------------------------------------------------ state
    def load(self, host: dict) -> None:
        """Uploads the host manager's state (``GpuExpertCache._export_slots``)."""
        self.slot_expert.copy_(host["slot_expert"])
        self.slot_gen.copy_(host["slot_gen"])
        self.slot_stamp.copy_(host["slot_stamp"])
        self.expert_slot.copy_(host["expert_slot"])
        self.clock.fill_(int(host["clock"]))
        self.counters.copy_(host["counters"])
        self.status.zero_()

    def read(self) -> dict:
        """The device state as host tensors (synchronises the stream)."""
        return dict(slot_expert=self.slot_expert.cpu(), slot_gen=self.slot_gen.cpu(),
                    slot_stamp=self.slot_stamp.cpu(), clock=int(self.clock.item()),
                    counters=self.counters.cpu(), status=int(self.status.item()))

    # ------------------------------------------------------------- work
    def plan(self, d, resident_first: bool, stream, later_waves: int = 0) -> None:
        """Plans every wave of the dispatch ``d``; with ``later_waves`` (a
        conditional handle of the graph being captured, ``capture_handle``)
        the plan also sets it to whether any wave after the first has
        experts."""
        N.check(N.lib.sf_dir_plan_ex(self.slot_expert.data_ptr(), self.slot_gen.data_ptr(),
                                     self.slot_stamp.data_ptr(), self.expert_slot.data_ptr(),
                                     self.clock.data_ptr(), self.counters.data_ptr(), d.active.data_ptr(),
                                     d.num_active.data_ptr(), self.E, self.S, self.waves, int(resident_first),
                                     self.wave_table.data_ptr(), self.wave_active.data_ptr(),
                                     self.wave_count.data_ptr(), self.fill_expert.data_ptr(),
                                     self.fill_slot.data_ptr(), self.fill_count.data_ptr(),
                                     self.status.data_ptr(), later_waves, stream), "sf_dir_plan")

    # ----------------------------------------------- captured later waves
    @staticmethod
    def capture_handle(stream) -> int:
        """A conditional handle of the graph ``stream`` is capturing into."""
        out = ctypes.c_uint64()
        N.check(N.lib.sf_capture_cond_handle(stream, ctypes.byref(out)), "sf_capture_cond_handle")
        return out.value

    @staticmethod
    def later_waves_stream(device) -> torch.cuda.ExternalStream:
        """The stream the later waves are captured on: the library's own
        per-device stream (not one of torch's pooled streams, which can be
        the very stream being captured)."""
        with torch.cuda.device(device):
            out = ctypes.c_void_p()
            N.check(N.lib.sf_capture_body_stream(ctypes.byref(out)), "sf_capture_body_stream")
        return torch.cuda.ExternalStream(out.value, device=device)

    def fill(self, wave: int, storage: torch.Tensor, stream) -> None:
        N.check(N.lib.sf_dir_fill(self.src_addr.data_ptr(), storage.data_ptr(),
                                  storage.stride(0) * storage.element_size(), self.expert_bytes,
                                  self.fill_expert[wave].data_ptr(), self.fill_slot[wave].data_ptr(),
                                  self.fill_count[wave:wave + 1].data_ptr(), self.S, self.fill_grid, stream),
                "sf_dir_fill")
