#!/usr/bin/env python3
"""Headline benchmark: copy GB/s (read + write) of the DataCopyExt strided gather on B200.

Workload: fp32 source [4096, 4096]; copy the column slab
[all rows, cols 1024..2047] into a contiguous [4096, 1024] destination, i.e.
DataCopyExt{blockCount=4096, blockLen=128x32 B, srcStride=384x32 B, dstStride=0}.
Algorithmic bytes per gather: 16 MiB read + 16 MiB written.

One *step* gathers from each of 16 rotating buffer sets (512 MiB touched per
step, > the 126 MB L2), so every launch reads cold data; the step's 16 launches
are captured once in a CUDA graph and the graph is replayed K times between two
CUDA events on the launching stream (host launch overhead stays out of the
device timing).  `value` = bytes moved by all ranks / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dcopy|reference]

`--impl reference` times the reference's CPU path instead: the C restatement of
its tiling semantics (oracle/, the reference's Ascend C CPU-debug build cannot
be built offline) on all host threads, same workload and metric.
Multi-GPU (torchrun): one rank per GPU, every rank runs the same workload on its
own GPU with no data-path collective (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "data-copy_b200"))
sys.path.insert(0, str(ROOT))

MIB = 1 << 20
ROWS, COLS, C0, C1 = 4096, 4096, 1024, 2048
BLOCK_LEN = (C1 - C0) * 4          # 4096 B = 128 x 32 B
SRC_GAP = (COLS - (C1 - C0)) * 4   # 12288 B = 384 x 32 B
BYTES_PER_GATHER = 2 * ROWS * BLOCK_LEN  # 16 MiB read + 16 MiB written
SETS = 16
METRIC = "copy GB/s (R+W) vs 8 TB/s HBM peak by burst/stride; aggregate at 1/2/4/8 GPUs"
WORKLOAD = ("config2_strided_gather: fp32 [4096,4096] cols 1024..2047 -> [4096,1024]; "
            "DataCopyExt blockCount=4096 blockLen=128x32B srcStride=384x32B dstStride=0")
NVML_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
                0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
                0x100: "display_clock_setting"}


def workload_config(world: int) -> dict:
    """The `config` object of both arms' JSON lines (the same keys and values)."""
    return {"workload": WORKLOAD, "gathers_per_step": SETS,
            "bytes_per_gather": BYTES_PER_GATHER,
            "l2": "inputs larger than L2: 16 rotating buffer sets, 512 MiB touched per step "
                  "vs 126 MB L2",
            "timing": "CUDA graph of one step replayed K times between CUDA events",
            "parallelism": f"independent per-GPU copies x{world} (no collective)"}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["dcopy", "reference"], default="dcopy")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the secondary measurements (sweep, NZ, transpose)")
    ap.add_argument("--workload", choices=["config2", "config4", "config5"], default="config2",
                    help="config2 (headline, default), config4 (ND<->NZ with batches split over "
                         "ranks) or config5 (sharded copy + NVLink ring)")
    return ap.parse_args()


# ---------------------------------------------------------------------------- helpers

def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    def __init__(self, cuda_index: int, period_s: float = 0.002):
        self.samples = []  # (host time, SM MHz)
        self.window = None
        self.reasons = 0
        self.max_mhz = None
        self.ok = False
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            import torch
            p = torch.cuda.get_device_properties(cuda_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            try:  # NVML and CUDA may order devices differently: match by PCI address
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # NVML missing: clocks reported as unavailable
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append((time.perf_counter(),
                                     n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)))
                try:
                    r = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    r = n.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.reasons |= int(r)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def mark(self, t0, t1):
        """Host-time bounds of the timed region."""
        self.window = (t0, t1)

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"],
                    "samples": len(self.samples)}
        names = [v for k, v in NVML_REASONS.items() if self.reasons & k and k != 0x1]
        inside = [mhz for t, mhz in self.samples
                  if self.window and self.window[0] <= t <= self.window[1]]
        window = "timed region"
        if len(inside) < 3:  # very short timed region: use the loaded warm-up as well
            inside = [mhz for _, mhz in self.samples]
            window = "warm-up soak + timed region"
        return {"sm_mhz": statistics.median(inside), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(inside), "window": window}


def cpu_baseline_gather(seconds: float = 8.0, threads=None):
    """The oracle's DataCopyExt gap copy (C, pthreads) on config 2, host memory."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    threads = threads or os.cpu_count() or 1
    src = np.random.default_rng(1).random((ROWS, COLS), dtype=np.float32)
    dst = np.empty((ROWS, C1 - C0), dtype=np.float32)
    view = src[:, C0:]
    O.copy_ext(dst, view, ROWS, BLOCK_LEN, SRC_GAP, 0, threads=threads)  # warm-up
    ref = src[:, C0:C1]
    assert (dst == ref).all(), "oracle gather mismatch"
    reps, t0 = 0, time.perf_counter()
    while True:
        O.copy_ext(dst, view, ROWS, BLOCK_LEN, SRC_GAP, 0, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return BYTES_PER_GATHER * reps / el / 1e9, reps, el, threads


# ---------------------------------------------------------------------------- dcopy arm

def run_dcopy(args, rank, world, local_rank):
    import torch
    import dcopy

    torch.cuda.set_device(local_rank)
    dcopy.lib()
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        dist = dist_mod

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    g = torch.Generator(device=dev).manual_seed(1 + rank)
    base = torch.rand(ROWS, COLS, generator=g, device=dev)
    srcs = [base.clone() for _ in range(SETS)]
    dsts = [torch.empty(ROWS, C1 - C0, device=dev) for _ in range(SETS)]
    stream = torch.cuda.current_stream()

    def one_step():
        for i in range(SETS):
            dcopy.copy_ext_32b(dsts[i], srcs[i][:, C0:], ROWS, BLOCK_LEN // 32, SRC_GAP // 32, 0)

    # Correctness first: bit-exact against the strided view before anything is timed.
    one_step()
    torch.cuda.synchronize()
    ref = base[:, C0:C1].contiguous().view(torch.int32)
    for d in dsts:
        assert torch.equal(d.view(torch.int32), ref), "gather mismatch"

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        one_step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        # Untimed soak (~0.3 s of replays) so the clock record sees a loaded GPU.
        for _ in range(30):
            for _ in range(100):
                graph.replay()
            torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        ev1.synchronize()
        clk.mark(t0, time.perf_counter())
        barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    launches = args.steps * SETS
    bytes_rank = BYTES_PER_GATHER * launches
    value = bytes_rank * world / (ms_max / 1e3) / 1e9
    launch_ms = ms / launches
    achieved = BYTES_PER_GATHER / (launch_ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    # DRAM bytes of one launch from an ncu capture of this bench's own launches
    # (profiles/strided_copy_kernel_config2_traffic.md): a committed figure, since
    # the counters cannot be read without the profiler.
    traffic_rec = load_traffic().get("strided_copy_kernel/config2") or {}
    traffic = traffic_rec.get("traffic_bytes_per_launch")

    # End to end through the public call with host buffers (pinned source and
    # destination, every step). dcopy_copy_ext_staged: the copy engine gathers the
    # 4 KiB bursts host -> device in chunks (16 MiB cross PCIe, not the 64 MiB
    # source) into a 16 MiB staging ring, and the copy engine returns each staged
    # chunk to the host destination on a second stream while the next chunk is
    # gathered, so both PCIe directions are busy. Measured on B200: the whole
    # source in and the result out around a device gather 21.9 GB/s; the kernel
    # reading and writing host memory directly (zero-copy, reported beside) 50-57
    # GB/s; this path 74.8 GB/s against a measured duplex ceiling of 87.2 GB/s.
    e2e_steps = max(3, min(args.steps, 30))
    h_src = base.cpu().pin_memory()
    h_dst = torch.empty(ROWS, C1 - C0).pin_memory()
    staging = torch.empty(16 * MIB, dtype=torch.uint8, device=dev)
    ref_host = h_src[:, C0:C1].contiguous().view(torch.int32)

    def staged_step():
        dcopy.copy_ext_staged(h_dst, h_src.data_ptr() + C0 * 4, ROWS, BLOCK_LEN, SRC_GAP, 0,
                              staging, flags=dcopy.STAGED_COPY_ENGINE_RETURN)

    def zero_copy_step():
        dcopy.copy_ext_32b(h_dst, h_src[:, C0:], ROWS, BLOCK_LEN // 32, SRC_GAP // 32, 0)

    def time_e2e(step):
        h_dst.fill_(float("nan"))
        for _ in range(2):
            step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            step()
        e1.record(stream)
        e1.synchronize()
        assert torch.equal(h_dst.view(torch.int32), ref_host), "end-to-end result mismatch"
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return BYTES_PER_GATHER * e2e_steps * world / (float(te.item()) / 1e3) / 1e9

    e2e_value = time_e2e(staged_step)
    zero_copy_value = time_e2e(zero_copy_step)

    # The same public call issued as a throughput user would: consecutive steps are
    # independent copies, alternating between two streams, each stream with its own
    # staging buffer and destination, so one step's gather overlaps the previous
    # step's return instead of waiting for it.  Every step still moves its inputs
    # host -> device and its result device -> host inside the timed region.
    side = torch.cuda.Stream(dev)
    h_dst2 = torch.empty(ROWS, C1 - C0).pin_memory()
    staging2 = torch.empty(16 * MIB, dtype=torch.uint8, device=dev)
    lanes = ((stream, h_dst, staging), (side, h_dst2, staging2))

    def alternating_step(k):
        st, d, sg = lanes[k % 2]
        dcopy.copy_ext_staged(d, h_src.data_ptr() + C0 * 4, ROWS, BLOCK_LEN, SRC_GAP, 0, sg,
                              flags=dcopy.STAGED_COPY_ENGINE_RETURN, stream=st)

    def time_alternating():
        h_dst.fill_(float("nan"))
        h_dst2.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        for k in range(2):
            alternating_step(k)
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        side.wait_event(e0)
        for k in range(e2e_steps):
            alternating_step(k)
        stream.wait_stream(side)
        e1.record(stream)
        e1.synchronize()
        for d in (h_dst, h_dst2):
            assert torch.equal(d.view(torch.int32), ref_host), "end-to-end result mismatch"
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return BYTES_PER_GATHER * e2e_steps * world / (float(te.item()) / 1e3) / 1e9

    two_stream_value = time_alternating()
    pcie = pcie_ceiling(torch, dev, barrier, dist, world)

    # N > 1: BASELINE config 5's NVLink step as well -- every rank pushes a 1 GiB
    # shard into rank (r + 1) mod N over NVLink, every received shard checked whole.
    p2p = None
    if world > 1:
        p2p = ring_shift_measure(torch, dcopy, dev, rank, world, barrier, dist, args.steps)

    # The other configs are single-GPU measurements: taken on the N=1 run only, so
    # multi-GPU runs do not hold N GPUs while rank 0 alone measures them.
    secondary = None
    if not args.no_secondary and world == 1:
        secondary = run_secondary(torch, dcopy, dev)

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            v, reps, el, thr = cpu_baseline_gather()
            v1, reps1, el1, _ = cpu_baseline_gather(seconds=3.0, threads=1)
            cpu = {"value": round(v, 3), "unit": "GB/s", "cores": thr, "kind": "port",
                   "sample": f"config 2 gather on host memory, {reps} reps in {el:.1f} s "
                             f"(oracle/dcopy_oracle.c oracle_copy_ext_mt, {thr} threads)",
                   "one_thread": {"value": round(v1, 3), "unit": "GB/s", "cores": 1,
                                  "sample": f"the same gather, {reps1} reps in {el1:.1f} s"}}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (torch.rand fp32 from seed 1+rank; copies are value-agnostic)",
            "config": workload_config(world),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel": "strided_copy_kernel<uint4,4>",
                         "algorithmic_bytes": BYTES_PER_GATHER,
                         "traffic_read": traffic_rec.get("dram_read_bytes_per_launch"),
                         "traffic_write": traffic_rec.get("dram_write_bytes_per_launch"),
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum per launch, "
                                         "ncu --cache-control none over 8 consecutive launches of "
                                         "this bench (writes land as later write-backs), no "
                                         "scaling; from profiles/ncu_traffic.json",
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(two_stream_value, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": ROWS * (C1 - C0) * 4,
                    "d2h_bytes_per_step": ROWS * (C1 - C0) * 4,
                    "steps": e2e_steps,
                    "path": "dcopy_copy_ext_staged on pinned host buffers, 16 MiB device "
                            "staging: copy-engine gather of the bursts host -> device in 6 "
                            "chunks, each chunk returned to host memory by the copy engine on "
                            "the library's return stream while the next is gathered; "
                            "consecutive steps (independent copies) alternate between two "
                            "caller streams, each with its own staging buffer and destination, "
                            "so a step's gather overlaps the previous step's return",
                    "serial_value": round(e2e_value, 3),
                    "serial_path": "the same call, every step on one stream (each step's "
                                   "pipeline fills and drains on its own)",
                    "pcie_duplex_ceiling_GBps": pcie["duplex"],
                    "pcie_h2d_GBps": pcie["h2d"], "pcie_d2h_GBps": pcie["d2h"],
                    "frac_of_duplex_ceiling": round(two_stream_value / world / pcie["duplex"], 4),
                    "pcie_note": "ceiling = 16 MiB pinned H2D and D2H cudaMemcpyAsync on two "
                                 "streams at once (per GPU); e2e moves the same bytes each way",
                    "zero_copy_value": round(zero_copy_value, 3),
                    "zero_copy_path": "dcopy_copy_ext_32b on the pinned host buffers: the kernel "
                                      "reads and writes host memory over PCIe"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if secondary is not None:
            line["secondary"] = secondary
        if p2p is not None:
            line["p2p"] = p2p
    return line


def pcie_ceiling(torch, dev, barrier, dist, world):
    """Per-GPU PCIe bandwidth of pinned 16 MiB cudaMemcpyAsync: host -> device alone,
    device -> host alone, and both at once on two streams (the duplex ceiling of an
    end-to-end copy, which moves the same bytes in each direction)."""
    n = 16 * MIB
    h_a = torch.empty(n, dtype=torch.uint8).pin_memory()
    h_b = torch.empty(n, dtype=torch.uint8).pin_memory()
    d_a = torch.empty(n, dtype=torch.uint8, device=dev)
    d_b = torch.empty(n, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream(dev)

    def run(h2d, d2h, reps=16):
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(main)
        s1.wait_event(a)
        s2.wait_event(a)
        for _ in range(reps):
            if h2d:
                with torch.cuda.stream(s1):
                    d_a.copy_(h_a, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s2):
                    h_b.copy_(d_b, non_blocking=True)
        main.wait_stream(s1)
        main.wait_stream(s2)
        b.record(main)
        b.synchronize()
        t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return round(n * reps * (int(h2d) + int(d2h)) / (float(t.item()) / 1e3) / 1e9, 2)

    run(True, True, reps=2)  # warm-up
    return {"h2d": run(True, False), "d2h": run(False, True), "duplex": run(True, True)}


def ring_shift_measure(torch, dcopy, dev, rank, world, barrier, dist, steps):
    """BASELINE config 5's exchange step on N GPUs: rank r pushes a 1 GiB shard into
    rank (r+1) mod N's receive buffer over NVLink (dcopy_p2p_copy into the CUDA IPC
    mapping), release-stores a sequence number into that rank's flag, and waits for
    its own flag with a bounded device-side wait.  Every received shard is compared
    whole with the sender's data.  Four runs on the same buffers: dcopy_p2p_copy
    with its automatic engine choice (the reported path), the same call with the SM
    engine forced (the bulk-copy push kernel), cudaMemcpyAsync in place of
    dcopy_p2p_copy, and NCCL send/recv of the same shards (the comparators).
    Timing: CUDA events on each rank's stream, max over ranks."""
    from dcopy import multi
    from cuda.bindings import runtime as cudart
    shard = 1 << 30
    words = shard // 4
    prev = (rank - 1) % world

    def pattern(r):  # the shard rank r sends: random words from seed 3 + r (BASELINE seed 3)
        g = torch.Generator(device=dev).manual_seed(3 + r)
        return torch.randint(-2**31, 2**31 - 1, (words,), dtype=torch.int32, device=dev,
                             generator=g)

    send = pattern(rank)
    expect = pattern(prev)
    recv = torch.zeros(words, dtype=torch.int32, device=dev)
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    barrier()
    peer = multi.map_next_peer(recv, flags, rank, world)
    seq = 0
    results = {}
    try:
        nxt = (rank + 1) % world

        def exchange(engine):
            nonlocal seq
            seq += 1
            if engine == "nccl":
                # NCCL send/recv of the same shards: the current stream waits for
                # NCCL's stream, so the events below bracket the transfer.
                ops = [dist.P2POp(dist.isend, send, nxt), dist.P2POp(dist.irecv, recv, prev)]
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
                return
            if engine == "copy_engine":
                err, = cudart.cudaMemcpyAsync(peer.recv_ptr, send.data_ptr(), shard,
                                              cudart.cudaMemcpyKind.cudaMemcpyDefault,
                                              stream.cuda_stream)
                if err != cudart.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaMemcpyAsync to the peer failed: {err}")
                dcopy.signal(peer.flag_ptr, seq, stream)
            else:
                multi.ring_shift(send, shard, peer, seq, stream)
            multi.wait_ring(flags, seq, status, timeout_ns=2_000_000_000, stream=stream)

        psteps = max(2, min(steps, 10))
        for name in ("dcopy", "sm_push", "copy_engine", "nccl"):
            prev_engine = dcopy.set_p2p_engine(
                dcopy.P2P_ENGINE_SM if name == "sm_push" else dcopy.P2P_ENGINE_AUTO)
            engine = name
            recv.zero_()
            barrier()
            for _ in range(2):
                exchange(engine)
            torch.cuda.synchronize(dev)
            ok = status.item() == 0 and torch.equal(recv, expect)
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(psteps):
                exchange(engine)
            e1.record(stream)
            e1.synchronize()
            ok = ok and status.item() == 0
            # The last exchange must also have delivered the whole shard.
            barrier()
            ok = ok and torch.equal(recv, expect)
            t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
            good = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.all_reduce(good, op=dist.ReduceOp.MIN)
            results[name] = (shard * psteps / (float(t.item()) / 1e3) / 1e9, bool(good.item()))
            dcopy.set_p2p_engine(prev_engine)
        err = dcopy.p2p_error()
    finally:
        barrier()
        peer.release()
    main, sm, ce, nc = (results["dcopy"], results["sm_push"], results["copy_engine"],
                        results["nccl"])
    return {"per_direction_GBps": round(main[0], 1), "aggregate_GBps": round(main[0] * world, 1),
            "nominal_GBps": 900.0, "frac_of_nominal": round(main[0] / 900.0, 4),
            "measured_peer_copy_GBps": 770.0,
            "frac_of_measured_peer_copy": round(main[0] / 770.0, 4),
            "flags_ok": main[1] and sm[1] and ce[1] and nc[1] and err == 0,
            "shards_checked": "whole 1 GiB shard, every run",
            "sm_push_per_direction_GBps": round(sm[0], 1),
            "copy_engine_per_direction_GBps": round(ce[0], 1),
            "nccl_send_recv_per_direction_GBps": round(nc[0], 1),
            "bytes_per_rank_per_step": shard, "steps": max(2, min(steps, 10)),
            "path": "dcopy_p2p_copy, automatic engine (pushes on the copy engine) "
                    "into the next rank's IPC-mapped buffer + release-store flag kernel; "
                    "bounded device-side wait kernel on this rank's flag",
            "sm_push_path": "the same with dcopy_set_p2p_engine(SM): p2p_bulk_push_kernel",
            "comparator": "cudaMemcpyAsync in place of dcopy_p2p_copy, same flags; and NCCL "
                          "send/recv (batch_isend_irecv) of the same shards"}


def _time_graph(torch, fn, reps=10, warm=3):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        fn()
    for _ in range(warm):
        g.replay()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(reps):
        g.replay()
    b.record(s)
    b.synchronize()
    return a.elapsed_time(b) / reps


def run_secondary(torch, dcopy, dev):
    """Short measurements of the other BASELINE configs (GB/s, R+W, one GPU)."""
    out = {}
    # Config 3 sweep: 256 MiB moved per point (> L2); int32 index-filled source.
    sweep = {}
    moved = 256 * MIB
    src = torch.empty((moved * 17) // 4, dtype=torch.int32, device=dev)
    dst = torch.empty(moved // 4, dtype=torch.int32, device=dev)
    for blen in (32, 64, 128, 512, 4096, 65536):
        for gx in (0, 1, 4, 16):
            count = moved // blen
            ms = _time_graph(torch, lambda: dcopy.copy_ext(dst, src, count, blen, gx * blen, 0),
                             reps=5, warm=2)
            sweep[f"{blen}B_gap{gx}x"] = round(2 * moved / (ms / 1e3) / 1e9, 1)
    out["config3_sweep_GBps"] = sweep
    del src, dst
    # Config 4: ND<->NZ fp16 [16, 4096, 4096] (512 MiB each way, > L2).
    shape = [16, 4096, 4096]
    nd = torch.empty(shape, dtype=torch.float16, device=dev).normal_()
    nz = torch.empty(16, 256, 256, 16, 16, dtype=torch.float16, device=dev)
    nbytes = nd.numel() * 2
    ms = _time_graph(torch, lambda: dcopy.nd_to_nz(nz, nd, shape, 2, 16), reps=10)
    ms2 = _time_graph(torch, lambda: dcopy.nz_to_nd(nd, nz, shape, 2, 16), reps=10)
    out["config4_nd_to_nz_GBps"] = round(2 * nbytes / (ms / 1e3) / 1e9, 1)
    out["config4_nz_to_nd_GBps"] = round(2 * nbytes / (ms2 / 1e3) / 1e9, 1)
    # The sibling tile format on the same tensor: ND<->FRACTAL_ZZ, c0 = 16.
    zz = nz.view(16, 256, 256, 16, 16)
    ms = _time_graph(torch, lambda: dcopy.nd_to_zz(zz, nd, shape, 2, 16), reps=10)
    ms2 = _time_graph(torch, lambda: dcopy.zz_to_nd(nd, zz, shape, 2, 16), reps=10)
    out["config4_nd_to_zz_GBps"] = round(2 * nbytes / (ms / 1e3) / 1e9, 1)
    out["config4_zz_to_nd_GBps"] = round(2 * nbytes / (ms2 / 1e3) / 1e9, 1)
    del nd, nz, zz
    # FRACTAL_Z (convolution weights): fp16 [2048, 2048, 3, 3], 72 MiB each way; two
    # weight/FRACTAL_Z pairs alternate so the working set (288 MiB) exceeds L2.
    n, c, h, w = 2048, 2048, 3, 3
    wts = [torch.empty(n * c * h * w, dtype=torch.float16, device=dev).normal_()
           for _ in range(2)]
    fzs = [torch.empty(c // 16 * h * w * n * 16, dtype=torch.float16, device=dev)
           for _ in range(2)]
    fzb = 2 * wts[0].numel() * 2
    frz = {}
    for name, fmt, shape in (("NCHW", 0, [n, c, h, w]), ("NHWC", 1, [n, h, w, c]),
                             ("HWCN", 16, [h, w, c, n])):
        def to_fz():
            for i in range(2):
                dcopy.to_fractal_z(fzs[i], wts[i], fmt, shape, 2, 16)

        def from_fz():
            for i in range(2):
                dcopy.from_fractal_z(wts[i], fzs[i], fmt, shape, 2, 16)
        ms = _time_graph(torch, to_fz, reps=10) / 2
        ms2 = _time_graph(torch, from_fz, reps=10) / 2
        frz[name] = [round(fzb / (ms / 1e3) / 1e9, 1), round(fzb / (ms2 / 1e3) / 1e9, 1)]
    out["fractal_z_fp16_2048x2048x3x3_to_from_GBps"] = frz
    del wts, fzs
    # The same weights as int8 with C0 = 32 (the 32-bit word paths for NCHW).
    wts8 = [torch.randint(0, 256, (n * c * h * w,), dtype=torch.uint8, device=dev)
            for _ in range(2)]
    fzs8 = [torch.empty(c // 32 * h * w * n * 32, dtype=torch.uint8, device=dev)
            for _ in range(2)]
    fzb8 = 2 * wts8[0].numel()
    frz8 = {}
    for name, fmt, shape in (("NCHW", 0, [n, c, h, w]), ("NHWC", 1, [n, h, w, c]),
                             ("HWCN", 16, [h, w, c, n])):
        def to_fz8():
            for i in range(2):
                dcopy.to_fractal_z(fzs8[i], wts8[i], fmt, shape, 1, 32)

        def from_fz8():
            for i in range(2):
                dcopy.from_fractal_z(wts8[i], fzs8[i], fmt, shape, 1, 32)
        ms = _time_graph(torch, to_fz8, reps=10) / 2
        ms2 = _time_graph(torch, from_fz8, reps=10) / 2
        frz8[name] = [round(fzb8 / (ms / 1e3) / 1e9, 1), round(fzb8 / (ms2 / 1e3) / 1e9, 1)]
    out["fractal_z_int8_2048x2048x3x3_to_from_GBps"] = frz8
    del wts8, fzs8
    # Standalone transpose at the 64 MiB maximum (rows 4088 x cols 4104 int32).
    rows, cols = 4088, 4104
    x = torch.empty(rows * cols, dtype=torch.int32, device=dev)
    ys = [torch.empty_like(x) for _ in range(4)]
    t = dcopy.plan_tiling(rows, cols, 240, 1)
    xs = [x] + [torch.empty_like(x) for _ in range(3)]

    def four():
        for i in range(4):
            dcopy.datacopy_large(xs[i], ys[i], t)
    ms = _time_graph(torch, four, reps=5) / 4
    out["standalone_large_64MiB_GBps"] = round(2 * x.numel() * 4 / (ms / 1e3) / 1e9, 1)
    # Config 1: contiguous fp16 512 KiB (L2-resident: latency, not bandwidth).
    # 16 copies per graph so the graph launch itself is not what is timed.
    a = [torch.empty(262144, dtype=torch.float16, device=dev) for _ in range(16)]
    b = [torch.empty_like(x) for x in a]

    def sixteen():
        for i in range(16):
            dcopy.copy_ext_32b(b[i], a[i], 128, 128, 0, 0)
    ms = _time_graph(torch, sixteen, reps=50) / 16
    out["config1_contiguous_512KiB_us"] = round(ms * 1e3, 2)
    # Config 1 with the reference's own structure: 8 cores x 16 tiles, one 4 KiB
    # DataCopy per tile -- 128 calls, or one dcopy_copy_ext_batch of 128 copies.
    x, y = a[0], b[0]
    tiles = [(y[i * 2048:], x[i * 2048:], 1, 4096, 0, 0) for i in range(128)]

    def per_tile():
        for (d, s, n_, l_, g1, g2) in tiles:
            dcopy.copy_ext(d, s, n_, l_, g1, g2)
    out["config1_128_tile_calls_us"] = round(_time_graph(torch, per_tile, reps=20) * 1e3, 2)
    out["config1_128_tiles_one_batch_us"] = round(
        _time_graph(torch, lambda: dcopy.copy_ext_batch(tiles), reps=50) * 1e3, 2)
    del a, b
    # Config 2's 16 gathers of one step as a single batch (one launch instead of 16).
    base = torch.empty(ROWS, COLS, device=dev)
    srcs = [torch.empty_like(base) for _ in range(SETS)]
    dsts = [torch.empty(ROWS, C1 - C0, device=dev) for _ in range(SETS)]
    gathers = [(dsts[i], srcs[i][:, C0:], ROWS, BLOCK_LEN, SRC_GAP, 0) for i in range(SETS)]
    ms = _time_graph(torch, lambda: dcopy.copy_ext_batch(gathers), reps=20)
    out["config2_16_gathers_one_batch_GBps"] = round(
        BYTES_PER_GATHER * SETS / (ms / 1e3) / 1e9, 1)
    return out


# ---------------------------------------------------------------------------- config 5

def run_config5(args, rank, world, local_rank):
    """bf16 8 x 1 GiB, blockCount split over ranks for the local
    strided copy (blockLen 2 KiB, gap 2 KiB), then a ring shift of each rank's
    1 GiB shard to rank (r+1) mod N over NVLink (CUDA IPC, in-kernel stores)."""
    import torch
    import dcopy
    torch.cuda.set_device(local_rank)
    dcopy.lib()
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        dist = dist_mod
    gib = 1 << 30
    blen = gap = 2048
    total_blocks = 8 * gib // (blen + gap)
    b0, nb = dcopy.shard_range(total_blocks, rank, world)
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    src = torch.empty(nb * (blen + gap) // 2, dtype=torch.bfloat16, device=dev)
    src.view(torch.int16).random_(generator=g)
    dst = torch.empty(nb * blen // 2, dtype=torch.bfloat16, device=dev)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    dcopy.copy_ext(dst, src, nb, blen, gap, 0)
    torch.cuda.synchronize()
    assert torch.equal(dst.view(torch.int16).view(nb, blen // 2),
                       src.view(torch.int16).view(nb, (blen + gap) // 2)[:, : blen // 2])
    for _ in range(max(args.warmup, 3)):
        dcopy.copy_ext(dst, src, nb, blen, gap, 0)
    barrier()
    steps = max(1, min(args.steps, 50))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dcopy.copy_ext(dst, src, nb, blen, gap, 0)
    e1.record()
    e1.synchronize()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    local_bytes = 2 * (total_blocks * blen)  # all ranks: 4 GiB read + 4 GiB written
    local_value = local_bytes * steps / (float(t.item()) / 1e3) / 1e9
    del src

    p2p = None
    if world > 1:  # the ring shift, every received 1 GiB shard checked whole
        p2p = ring_shift_measure(torch, dcopy, dev, rank, world, barrier, dist, args.steps)
    if rank != 0:
        return None
    return {"metric": METRIC, "value": round(local_value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(float(t.item()) / steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random bf16 bit patterns from seed 3+rank)",
            "config": {"workload": "config5: bf16 8 x 1 GiB, blockLen 2 KiB, srcStride gap 2 KiB, "
                                   "blockCount split over ranks; ring shift of 1 GiB per rank",
                       "blocks_per_rank": nb, "l2": "inputs larger than L2 (8/N GiB per rank)"},
            "p2p": p2p}


# ---------------------------------------------------------------------------- config 4

def run_config4(args, rank, world, local_rank):
    """BASELINE config 4 on N GPUs: fp16 [16, 4096, 4096] ND -> FRACTAL_NZ -> ND, the 16
    batches (the `times` axis, outermost on both sides) split over ranks with no
    exchange (strong scaling); every rank times its own round trips, max over ranks."""
    import torch
    import dcopy
    torch.cuda.set_device(local_rank)
    dcopy.lib()
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        dist = dist_mod
    T, H, W = 16, 4096, 4096
    b0, nb = dcopy.shard_range(T, rank, world)
    batch_bytes = H * W * 2
    # Enough buffer sets that each rank's working set exceeds L2 (>= 512 MiB).
    sets = max(1, min(4, -(-(512 * MIB) // max(1, 2 * nb * batch_bytes))))
    g = torch.Generator(device=dev).manual_seed(2)
    nds = [torch.empty(nb, H, W, dtype=torch.float16, device=dev) for _ in range(sets)]
    for x in nds:
        x.normal_(generator=g)
    nzs = [torch.empty(nb, W // 16, H // 16, 16, 16, dtype=torch.float16, device=dev)
           for _ in range(sets)]
    shape = [nb, H, W]

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def step():
        for i in range(sets):
            dcopy.nd_to_nz(nzs[i], nds[i], shape, 2, 16)
        for i in range(sets):
            dcopy.nz_to_nd(nds[i], nzs[i], shape, 2, 16)

    if nb:
        ref = nds[0].clone()
        step()
        torch.cuda.synchronize()
        want = ref.view(nb, H // 16, 16, W // 16, 16).permute(0, 3, 1, 2, 4)
        assert torch.equal(nzs[0].view(torch.int16), want.view(torch.int16)), "ND->NZ mismatch"
        assert torch.equal(nds[0].view(torch.int16), ref.view(torch.int16)), "NZ->ND mismatch"
        del ref, want
        for _ in range(max(args.warmup, 3)):
            step()
    barrier()
    steps = max(1, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps if nb else 0):
        step()
    e1.record()
    e1.synchronize()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    # All ranks together: every batch read and written once per direction per set.
    total_bytes = 2 * 2 * T * batch_bytes * sets * steps
    value = total_bytes / (float(t.item()) / 1e3) / 1e9
    if rank != 0:
        return None
    return {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(float(t.item()) / steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (normal(0,1) fp16 from seed 2)",
            "config": {"workload": "config4: fp16 [16,4096,4096] ND -> FRACTAL_NZ [16,256,256,16,16]"
                                   " -> ND, batches split over ranks",
                       "batches_per_rank0": nb, "buffer_sets": sets,
                       "l2": "each rank's working set >= 512 MiB (rotating buffer sets)"}}


# ---------------------------------------------------------------------------- reference arm

def run_reference(args):
    threads = os.cpu_count() or 1
    import numpy as np
    from oracle import oracle as O
    O.build()
    src = np.random.default_rng(1).random((ROWS, COLS), dtype=np.float32)
    dst = np.empty((ROWS, C1 - C0), dtype=np.float32)
    view = src[:, C0:]
    for _ in range(max(args.warmup, 3)):
        O.copy_ext(dst, view, ROWS, BLOCK_LEN, SRC_GAP, 0, threads=threads)
    assert (dst == src[:, C0:C1]).all()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.copy_ext(dst, view, ROWS, BLOCK_LEN, SRC_GAP, 0, threads=threads)
    el = time.perf_counter() - t0
    value = BYTES_PER_GATHER * args.steps / el / 1e9
    sample = (f"full config 2 gather per step on host memory (oracle_copy_ext_mt, the C "
              f"restatement of the reference's DataCopyExt semantics), {threads} threads")
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return 0
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        # NCCL writes its debug output, the version banner included (printed at the
        # VERSION and WARN levels), to stdout unless NCCL_DEBUG_FILE names a file;
        # rank 0's stdout must carry exactly one JSON line.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "config5":
            line = run_config5(args, rank, world, local_rank)
        elif args.workload == "config4":
            line = run_config4(args, rank, world, local_rank)
        else:
            line = run_dcopy(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
