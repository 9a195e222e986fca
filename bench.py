# SPDX-License-Identifier: Apache-2.0
"""Paged-attention decode benchmark (one JSON line on rank 0).

Workload (default): continuous-batching decode at Llama-3-8B attention shape,
32 q / 8 kv heads, head_dim 128, 32 layers, MX-FP8 KV in 16-token pages,
256 requests with log-uniform contexts in [128, 16384], blocks scattered over
an arena. One step = the 32 layers' decode attention of every request (one
launch per layer, as a model runs it). Requests are sharded over N GPUs by
longest-processing-time packing, with no communication (strong scaling:
the batch is fixed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kllm|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the reference's own CPU attention
(userspace/compute/ace_attention.c, built from its sources into oracle/_ref)
on the host cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import select
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "xpu-kllm_b200"))

from kllm_b200 import multigpu as mg  # noqa: E402
from kllm_b200 import workloads as wl  # noqa: E402

METRIC = "paged-attn decode KV GB/s (% of 8 TB/s HBM) & tokens/s at 1/2/4/8 B200"

# DRAM bytes per decode launch / algorithmic bytes, from an ncu capture of
# two decode_kernel<128,1> launches of the C3 workload itself (every launch
# covers the full 256-request batch of one layer, 1.8273 GB algorithmic):
# 1,830.7 + 4.9 MB and 1,830.6 + 2.6 MB read + written. Other decode
# workloads scale it by the bytes they process.
DECODE_TRAFFIC_RATIO = 1.0038

# What the decode computes in, per KV format: MX-FP8 pages are dequantised in
# registers to f16 (exact E4M3 x E4M3 products, scaled by 2^-2) and contracted
# by f16 tensor-core MMAs with fp32 accumulation; BF16 pages by bf16 MMAs.
DECODE_DTYPE = {wl.KV_MX_FP8: "f16 MMA, fp32 accum (MX-FP8 E4M3 KV dequantised in registers)",
                wl.KV_BF16: "bf16 MMA, fp32 accum (BF16 KV)"}


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and clock-event-reason samples during the timed region: NVML
    read every 10 ms from a thread (so that regions of a few milliseconds
    still get samples), else nvidia-smi every 100 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int, period: float = 0.01):
        self.index = index
        self.period = period
        self.proc = None
        self.thread = None

    def _nvml_start(self) -> bool:
        try:
            import threading
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return False
        self.samples, self.stop_ev = [], threading.Event()

        def run():
            while True:
                try:
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         mx, int(reasons(h))))
                except Exception:
                    pass
                if self.stop_ev.wait(self.period):
                    break
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        return True

    def start(self):
        if self._nvml_start():
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        # wait (up to 3 s) for the first sample, so that the sampler is
        # running when the timed region starts; that sample is taken before
        # the region and is not counted
        ready, _, _ = select.select([self.proc.stdout], [], [], 3.0)
        if ready:
            self.proc.stdout.readline()

    def stop(self) -> dict:
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            sm = [float(x[0]) for x in self.samples]
            mx = [float(x[1]) for x in self.samples]
            reasons = {nm for x in self.samples for nm, bit in self.BITS.items() if x[2] & bit}
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                    "samples": len(sm), "source": "nvml, 10 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 100 ms"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

class DecodeRig:
    """The rank's requests resident on its GPU: pages, table, Q, outputs."""

    def __init__(self, cfg: wl.DecodeConfig, seqs: list[int], all_lens: np.ndarray, be,
                 torch, device: int, seed: int = 0, arena_factor: float = 1.25,
                 layer_major: bool = True):
        self.cfg, self.be, self.torch = cfg, be, torch
        self.seqs = seqs
        self.lens = np.asarray(all_lens)[seqs].astype(np.int32)
        c = cfg
        self.B = len(seqs)
        dev = torch.device("cuda", device)
        pages = (self.lens.astype(np.int64) + c.block - 1) // c.block
        need = int(pages.sum())
        free, _ = torch.cuda.mem_get_info(device)
        slot_b = c.slot_bytes()
        want = int(math.ceil(need * arena_factor))
        cap = int((free * 0.85 - 4e9) // slot_b)
        n_slots = max(need, min(want, cap))
        self.arena_bytes = n_slots * slot_b
        self.plan = wl.plan_pages(c, self.lens, seed, n_slots=n_slots)
        self.arena = torch.empty(self.arena_bytes, dtype=torch.uint8, device=dev)
        # layer-major: layer l of every slot is one contiguous region, so a
        # launch (one layer) touches n_slots x 36 KB instead of 36 KB in each
        # 1.18 MB all-layer slot (far fewer GPU pages per launch)
        self.layer_major = layer_major
        self.slot_pitch = c.layer_stride() if layer_major else slot_b
        self.layer_stride = n_slots * c.layer_stride() if layer_major else c.layer_stride()
        table = wl.block_table(self.plan, c, self.arena.data_ptr(), slot_pitch=self.slot_pitch)
        self.table = torch.from_numpy(table.view(np.uint8).copy()).to(dev)
        self.seq_lens = torch.from_numpy(self.lens.copy()).to(dev)
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000003 + 17)
        mult = torch.from_numpy(wl.magnitudes(c, seed)[seqs].astype(np.float32)).to(dev)
        self.q = torch.randn((c.layers, self.B, c.hq, c.d), generator=g, device=dev,
                             dtype=torch.float32).to(torch.bfloat16)
        self.out = torch.zeros((c.layers, self.B, c.hq, c.d), dtype=torch.bfloat16, device=dev)
        self._fill(g, mult, dev)

    def _fill(self, g, mult, dev):
        """Quantize-on-write of every context token through the append ABI."""
        torch, c = self.torch, self.cfg
        st = torch.cuda.current_stream().cuda_stream
        chunk = 1 << 17
        tok_seq = np.concatenate([np.full(L, i, np.int32) for i, L in enumerate(self.lens)])
        tok_pos = np.concatenate([np.arange(L, dtype=np.int32) for L in self.lens])
        ts_all = torch.from_numpy(tok_seq).to(dev)
        tp_all = torch.from_numpy(tok_pos).to(dev)
        for layer in range(c.layers):
            for a in range(0, len(tok_seq), chunk):
                b = min(a + chunk, len(tok_seq))
                ts, tp = ts_all[a:b], tp_all[a:b]
                m = mult[ts.long()][:, :, None]
                k = (torch.randn((b - a, c.hkv, c.d), generator=g, device=dev) * m).to(
                    torch.bfloat16)
                v = (torch.randn((b - a, c.hkv, c.d), generator=g, device=dev) * m).to(
                    torch.bfloat16)
                rc = self.be.append(k=k.data_ptr(), v=v.data_ptr(), token_seq=ts.data_ptr(),
                                    token_pos=tp.data_ptr(), num_tokens=b - a,
                                    num_seqs=self.B,
                                    block_tables=self.table.data_ptr(),
                                    max_blocks_per_seq=self.plan.max_blocks,
                                    num_kv_heads=c.hkv, head_dim=c.d, block_size=c.block,
                                    kv_dtype=c.kv_dtype, layer=layer,
                                    layer_stride=self.layer_stride, stream=st)
                assert rc == 0, f"append failed: {rc}"
        torch.cuda.synchronize()

    split_kv = False
    entry = "context"   # "noalloc": kllm_gpu_paged_attention_v2_noalloc (no context workspace)
    # consecutive layers' decodes: each may start while the previous one
    # finishes (the block table and seq_lens are not written between them)
    flags = 0x1         # KLLM_DECODE_OVERLAP_PREV

    def enable_split_kv(self, rank: int, world: int, dist, merge: str = "p2p") -> None:
        """Cross-GPU split-KV: partial triples per rank, exchanged and merged
        inside every step, either by one peer-memory kernel per rank
        (kllm_gpu_p2p_merge) or over NCCL (kllm_gpu_comm_merge)."""
        import ctypes
        torch, c = self.torch, self.cfg
        rows = self.B * c.hq
        self.merge = merge
        if merge == "p2p":
            h = (ctypes.c_uint8 * 64)()
            rc = self.be.lib.kllm_gpu_p2p_export(self.be.ctx, rows, c.d, h)
            if rc != 0:
                raise RuntimeError(f"kllm_gpu_p2p_export: {rc}")
            mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device="cuda")
            allh = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allh, mine)
            blob = bytes(torch.cat(allh).cpu().tolist())
            rc = self.be.lib.kllm_gpu_p2p_import(self.be.ctx, world, rank,
                                                 (ctypes.c_uint8 * len(blob))(*blob))
            if rc != 0:
                raise RuntimeError(f"kllm_gpu_p2p_import: {rc}")
            self.p2p_err = torch.zeros(1, dtype=torch.int32, device="cuda")
        else:
            uid = (ctypes.c_uint8 * 128)()
            if rank == 0:
                rc = self.be.lib.kllm_gpu_comm_get_unique_id(uid)
                assert rc == 0, f"comm id: {rc}"
            t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device="cuda")
            dist.broadcast(t, 0)
            uid = (ctypes.c_uint8 * 128)(*t.cpu().tolist())
            rc = self.be.lib.kllm_gpu_comm_init(self.be.ctx, world, rank, uid, 120000)
            if rc != 0:
                raise RuntimeError(f"kllm_gpu_comm_init: {rc}")
        self.pm = torch.empty((rows,), dtype=torch.float32, device="cuda")
        self.pl = torch.empty_like(self.pm)
        self.po = torch.empty((rows, c.d), dtype=torch.float32, device="cuda")
        self.split_kv = True

    def launch(self, layer: int, stream: int, q_ptr=None, out_ptr=None) -> None:
        c = self.cfg
        kw = dict(
            output=out_ptr or self.out[layer].data_ptr(),
            query=q_ptr or self.q[layer].data_ptr(),
            block_tables=self.table.data_ptr(), seq_lens=self.seq_lens.data_ptr(),
            num_seqs=self.B, num_heads=c.hq, num_kv_heads=c.hkv, head_dim=c.d,
            max_blocks_per_seq=self.plan.max_blocks, block_size=c.block, kv_dtype=c.kv_dtype,
            layer=layer, layer_stride=self.layer_stride, scale=c.scale, split=1, stream=stream,
            flags=self.flags)
        if self.split_kv:
            kw.update(output=None, partial_m=self.pm.data_ptr(), partial_l=self.pl.data_ptr(),
                      partial_o=self.po.data_ptr())
        if self.entry == "noalloc":
            import ctypes
            import kllm_b200 as kb
            p = kb.AttnParamsV2()
            p.struct_size = ctypes.sizeof(p)
            for k, v in kw.items():
                setattr(p, k, v)
            rc = self.be.lib.kllm_gpu_paged_attention_v2_noalloc(ctypes.byref(p))
        else:
            rc = self.be.decode_v2(**kw)
        if rc != 0:
            raise RuntimeError(f"decode launch failed: {rc}")
        if self.split_kv and self.merge == "p2p":
            rc = self.be.lib.kllm_gpu_p2p_merge(
                self.be.ctx, self.pm.data_ptr(), self.pl.data_ptr(), self.po.data_ptr(),
                self.B * c.hq, c.d, out_ptr or self.out[layer].data_ptr(),
                self.p2p_err.data_ptr(), 2000, stream)
            if rc != 0:
                raise RuntimeError(f"kllm_gpu_p2p_merge failed: {rc}")
        elif self.split_kv:
            rc = self.be.lib.kllm_gpu_comm_merge(
                self.be.ctx, self.pm.data_ptr(), self.pl.data_ptr(), self.po.data_ptr(),
                self.B * c.hq, c.d, out_ptr or self.out[layer].data_ptr(), stream, 0)
            if rc != 0:
                raise RuntimeError(f"kllm_gpu_comm_merge failed: {rc}")

    def step_bytes(self) -> int:
        return wl.algorithmic_bytes(self.cfg, self.lens)

    def host_sample(self, seqs_local: list[int], layer: int = 0):
        """Copies the sampled requests' pages of one layer to a compact host
        arena; returns (cfg1, lens, table rows over the host arena, arena)."""
        import dataclasses
        c = self.cfg
        c1 = dataclasses.replace(c, layers=1, batch=len(seqs_local))
        lens = self.lens[seqs_local]
        plan_rows = self.plan.slots[seqs_local]
        used = plan_rows[plan_rows >= 0]
        host = np.zeros((len(used), c1.slot_bytes()), dtype=np.uint8)
        arena_view = self.arena.view(-1)
        loff = layer * self.layer_stride
        remap = {}
        for i, sl in enumerate(used):
            a = int(sl) * self.slot_pitch + loff
            host[i] = arena_view[a:a + c.layer_stride()].cpu().numpy()
            remap[int(sl)] = i
        slots = np.full(plan_rows.shape, -1, np.int64)
        for r in range(plan_rows.shape[0]):
            for b in range(plan_rows.shape[1]):
                if plan_rows[r, b] >= 0:
                    slots[r, b] = remap[int(plan_rows[r, b])]
        plan = wl.PagePlan(seq_lens=lens, slots=slots, n_slots=len(used),
                           max_blocks=plan_rows.shape[1], pages_used=len(used))
        table = wl.block_table(plan, c1, host.ctypes.data)
        return c1, lens, table, host


def run_kllm(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    os.environ["KLLM_GPU_DEVICE"] = str(local)
    import kllm_b200 as kb
    be = kb.Backend()
    if be.backend != kb.KLLM_GPU_CUDA:
        raise RuntimeError("libkllm_gpu: no sm_100 device")
    # torch work (data generation, events) and the library's launches share
    # the context stream, so every CUDA event brackets the library's kernels
    torch.cuda.set_stream(be.torch_stream())

    cfg = wl.CONFIGS[args.config]
    if args.layers:
        cfg = __import__("dataclasses").replace(cfg, layers=args.layers)
    lens_all = wl.context_lengths(cfg, args.seed)
    split_kv = cfg.batch == 1 and world > 1
    if split_kv:
        # one long context: this rank owns a contiguous range of its pages
        pages = int((lens_all[0] + cfg.block - 1) // cfg.block)
        lo, hi = mg.page_ranges(pages, world)[rank]
        local_len = int(np.clip(lens_all[0] - lo * cfg.block, 0, (hi - lo) * cfg.block))
        mine, lens_rank = [0], np.array([local_len], np.int32)
    elif args.shard_of:
        # one rank's share of an N-way request split, timed alone on this GPU
        # (what each GPU of an N-GPU run does; no other rank exists)
        r_e, n_e = (int(x) for x in args.shard_of.split("/"))
        mine = mg.lpt_shard(lens_all, n_e)[r_e]
        lens_rank = lens_all
    else:
        mine = mg.lpt_shard(lens_all, world)[rank]
        lens_rank = lens_all
    rig = DecodeRig(cfg, mine, lens_rank, be, torch, local, args.seed,
                    layer_major=args.arena_layout == "layer-major")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    if split_kv:
        rig.enable_split_kv(rank, world, dist, args.merge)
    if args.decode_entry == "noalloc":
        if split_kv:
            raise SystemExit("--decode-entry noalloc times the single-GPU decode only")
        rig.entry = "noalloc"
        rig.flags = 0
    if args.no_overlap:
        rig.flags = 0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up
    for _ in range(args.warmup):
        for layer in range(cfg.layers):
            rig.launch(layer, sp)
    barrier()

    # device-timed region: KV (63 GB at 1 GPU) is far larger than the 126 MB L2
    clk = Clocks(local)
    clk.start()
    launches0 = be.stats().launches
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        for layer in range(cfg.layers):
            rig.launch(layer, sp)
    t1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = be.stats().launches - launches0
    elapsed_ms = t0.elapsed_time(t1)
    if rig.split_kv and rig.merge == "p2p" and int(rig.p2p_err.item()) != 0:
        raise RuntimeError(f"peer-memory exchange error word {int(rig.p2p_err.item()):#x}")
    # mean decode launch = the timed region / decode launches: only the decode
    # (and its merge, which is empty unless a segment has > 16 pieces) runs
    # there; an event pair around every launch would cost 1-4% by itself
    per_launch = [elapsed_ms / (args.steps * cfg.layers)]

    # end-to-end through the C ABI: pinned host Q in, bf16 O out, every step
    host_q = torch.empty_like(rig.q, device="cpu").pin_memory()
    host_q.copy_(rig.q.cpu())
    host_o = torch.empty_like(rig.out, device="cpu").pin_memory()
    host_lens = torch.from_numpy(rig.lens.copy()).pin_memory()
    lib, ctx = be.lib, be.ctx
    qb = rig.q[0].numel() * 2
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    # copies on their own streams (uploads, read-backs), overlapping the
    # decode of neighbouring layers; events order each layer's upload ->
    # decode -> read-back, and a layer's buffers are reused only after the
    # previous step's decode / read-back of that layer finished
    up_s, down_s = torch.cuda.Stream(), torch.cuda.Stream()
    L = cfg.layers
    ev_in = [torch.cuda.Event() for _ in range(L)]
    ev_done = [torch.cuda.Event() for _ in range(L)]
    ev_out = [torch.cuda.Event() for _ in range(L)]
    ev_go = torch.cuda.Event()
    ev_end = torch.cuda.Event()

    def e2e_step(first=False):
        lib.kllm_gpu_memcpy_h2d_async(ctx, rig.seq_lens.data_ptr(), host_lens.data_ptr(),
                                      host_lens.numel() * 4, sp)
        if first:                                    # no copy starts before the region opens
            ev_go.record(stream)
            up_s.wait_event(ev_go)
        for layer in range(L):
            up_s.wait_event(ev_done[layer])          # the previous step read q[layer]
            lib.kllm_gpu_memcpy_h2d_async(ctx, rig.q[layer].data_ptr(),
                                          host_q[layer].data_ptr(), qb, up_s.cuda_stream)
            ev_in[layer].record(up_s)
        for layer in range(L):
            stream.wait_event(ev_in[layer])
            stream.wait_event(ev_out[layer])         # the previous step's read-back of out
            rig.launch(layer, sp)
            ev_done[layer].record(stream)
            down_s.wait_event(ev_done[layer])
            lib.kllm_gpu_memcpy_d2h_async(ctx, host_o[layer].data_ptr(),
                                          rig.out[layer].data_ptr(), qb, down_s.cuda_stream)
            ev_out[layer].record(down_s)
        ev_end.record(down_s)
        stream.wait_event(ev_end)                    # the step ends with its last read-back

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i == 0)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if not torch.equal(host_o[L - 1][:4].to(rig.out.device), rig.out[L - 1][:4]):
        raise RuntimeError("end-to-end read-back differs from the device output")

    my_bytes = rig.step_bytes()
    stats = torch.tensor([elapsed_ms, e2e_ms, float(my_bytes), float(rig.B),
                          float(np.mean(per_launch)), float(rig.arena_bytes)],
                         dtype=torch.float64, device="cuda")
    if world > 1:
        gathered = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(gathered, stats)
        allst = torch.stack(gathered).cpu().numpy()
    else:
        allst = stats.cpu().numpy()[None]
    t_ms = float(allst[:, 0].max())
    te_ms = float(allst[:, 1].max())
    total_bytes = float(allst[:, 2].sum())
    total_tokens = float(cfg.batch) if split_kv else float(allst[:, 3].sum())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_from_rig(rig, args)
    per_req = None
    if args.per_request_compare and world == 1 and not split_kv:
        per_req = per_request_step_ms(rig, torch, max(1, min(args.steps, 3)))

    if world > 1:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = peaks()
        ms_step = t_ms / args.steps
        value = total_bytes * args.steps / (t_ms * 1e-3) / 1e9
        e2e_val = total_bytes * args.steps / (te_ms * 1e-3) / 1e9
        # roofline of the decode kernel: rank 0's algorithmic bytes per launch
        # over its mean CUDA-event launch time (burst peak: timed per launch)
        per_launch_bytes = float(allst[0, 2]) / cfg.layers
        achieved = per_launch_bytes / (float(allst[0, 4]) * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": DECODE_DTYPE[cfg.kv_dtype],
            "data": "synthetic (seeded; KV quantized on device by the append kernel)",
            "config": {"workload": cfg.name, "batch": cfg.batch, "layers": cfg.layers,
                       "hq": cfg.hq, "hkv": cfg.hkv, "head_dim": cfg.d, "block": cfg.block,
                       "kv_format": "mx-fp8-e4m3 (e4m3 scale per 8)",
                       "kv_gb_per_step": round(total_bytes / 1e9, 3),
                       "arena_gb_rank0": round(float(allst[0, 5]) / 1e9, 2),
                       "arena_layout": args.arena_layout,
                       "decode_launch": ("programmatic dependent of the previous layer's "
                                         "kernels (KLLM_DECODE_OVERLAP_PREV)" if rig.flags
                                         else "after the previous kernel completed"),
                       "l2": "inputs larger than L2 (KV per step >> 126 MB)",
                       "parallelism": ((f"split-KV x{world} (page ranges) + one peer-memory "
                                        f"exchange-and-merge kernel per rank (NVLink)"
                                        if args.merge == "p2p" else
                                        f"split-KV x{world} (page ranges) + NCCL all-gather "
                                        f"merge") if split_kv else
                                       f"request-sharded x{world} (LPT), no collective")},
            "tokens_per_s": round(total_tokens * args.steps / (t_ms * 1e-3), 1),
            "hbm_frac_8tbs": round(value / world / 8000.0, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind,
                         "traffic": round(per_launch_bytes * DECODE_TRAFFIC_RATIO),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                           "of two C3 decode launches (--layers 2): mean "
                                           "1,834.4 MB per launch against 1,827.3 MB "
                                           "algorithmic = 1.0038, times this launch's "
                                           "algorithmic bytes "
                                           "(profiles/launch_list_c3_decode_bench.md)",
                         "kernel": "decode_kernel<128,1> (MX-FP8)"},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(cfg.layers * qb + rig.B * 4),
                    "d2h_bytes_per_step": int(cfg.layers * qb)},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if args.decode_entry == "noalloc":
            line["config"]["decode_entry"] = "kllm_gpu_paged_attention_v2_noalloc"
        if args.shard_of:
            line["config"]["shard_of"] = (f"requests of rank {args.shard_of} (LPT) only, "
                                          f"on one GPU: value is that rank's share")
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if per_req is not None:
            line["per_request_launches"] = {
                "ms_per_step": round(per_req[0], 3), "launches_per_step": per_req[1],
                "batched_ms_per_step": round(ms_step, 4),
                "note": "the same step with one decode launch per request per layer, the "
                        "pattern of userspace/reactor/batch_scheduler.c:258-263"}
        print(json.dumps(line), flush=True)
        if cpu is not None and not cpu["gpu_matches_reference_on_sample"]:
            raise SystemExit("bench: the GPU decode of the sampled requests differs from the "
                             "reference CPU attention beyond 1e-3 + 2e-2|ref|")
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    be.close()
    if world > 1:
        dist.destroy_process_group()


def per_request_step_ms(rig, torch, steps: int):
    """(ms per step, launches per step) of the step issued one request at a
    time: every layer, every request gets its own decode launch (table row,
    seq_len, query and output rows of that request)."""
    c = rig.cfg
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    row_b = rig.plan.max_blocks * 24
    q_b = c.hq * c.d * 2

    def one_step():
        for layer in range(c.layers):
            for s in range(rig.B):
                rc = rig.be.decode_v2(
                    output=rig.out[layer].data_ptr() + s * q_b,
                    query=rig.q[layer].data_ptr() + s * q_b,
                    block_tables=rig.table.data_ptr() + s * row_b,
                    seq_lens=rig.seq_lens.data_ptr() + 4 * s, num_seqs=1, num_heads=c.hq,
                    num_kv_heads=c.hkv, head_dim=c.d, max_blocks_per_seq=rig.plan.max_blocks,
                    block_size=c.block, kv_dtype=c.kv_dtype, layer=layer,
                    layer_stride=rig.layer_stride, scale=c.scale, split=1, stream=sp)
                if rc != 0:
                    raise RuntimeError(f"decode launch failed: {rc}")
    one_step()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        one_step()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, c.layers * rig.B


def cpu_baseline_from_rig(rig, args) -> dict:
    """The reference CPU attention on a bounded sample of the GPU-resident
    workload (one layer of a subset of requests, pages copied back), timed on
    the host cores; also checks the GPU outputs of that sample."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    lib = oracle.ref()
    kind, prefix = ("reference", "ref") if lib is not None else ("port", "orc")
    if lib is None:
        lib = oracle.orc()
    order = np.argsort(rig.lens)
    pick = sorted(int(i) for i in order[np.linspace(0, len(order) - 1, 24).astype(int)])
    c1, lens, table, host = rig.host_sample(pick, layer=0)
    q = rig.q[0][pick].contiguous().view(rig.torch.int16).cpu().numpy().view(np.uint16)
    nthreads = os.cpu_count() or 1
    out, wall, g, a = oracle.harness_decode(lib, prefix, q, table, lens, c1.hq, c1.hkv, c1.d,
                                            table.shape[1], c1.scale, c1.block, c1.kv_dtype, 0,
                                            nthreads)
    reps, total = 1, wall
    while total < args.cpu_seconds and reps < 200:
        _, w2, _, _ = oracle.harness_decode(lib, prefix, q, table, lens, c1.hq, c1.hkv, c1.d,
                                            table.shape[1], c1.scale, c1.block, c1.kv_dtype, 0,
                                            nthreads)
        total += w2
        reps += 1
    sample_bytes = wl.algorithmic_bytes(c1, lens, layers=1)
    gpu = rig.out[0][pick].contiguous().view(rig.torch.int16).cpu().numpy().view(np.uint16)
    gf, rf = wl.bf16_to_f32(gpu), wl.bf16_to_f32(out)
    ok = bool(np.all(np.abs(gf - rf) <= 1e-3 + 2e-2 * np.abs(rf)))
    return {"value": round(sample_bytes * reps / total / 1e9, 3), "unit": "GB/s",
            "cores": nthreads, "kind": kind,
            "sample": f"layer 0 of {len(pick)} requests ({int(lens.sum())} tokens, "
                      f"{sample_bytes / 1e6:.1f} MB) x {reps} reps",
            "gather_dequant_s": round(g, 4), "attention_s": round(a, 4),
            "gpu_matches_reference_on_sample": ok}


# ---------------------------------------------------------------------------
# chunked prefill + KV append (C5)
# ---------------------------------------------------------------------------

PREFILL_METRIC = "chunked prefill + MX-FP8 KV append: prompt tokens/s (attention TFLOP/s)"


def bf16_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


class PrefillRig:
    """One layer of the C5 step resident on the GPU: the chunk's Q/K/V, the
    cache (with the shared prefix chain already written), table and outputs."""

    def __init__(self, cfg: wl.DecodeConfig, be, torch, device: int, seed: int = 0):
        self.cfg, self.be, self.torch = cfg, be, torch
        c = cfg
        dev = torch.device("cuda", device)
        self.ctx, self.chunk = wl.prefill_split(c)
        self.n_tok = int(self.chunk.sum())
        self.plan = wl.plan_prefill_pages(c, self.ctx, self.chunk, seed)
        self.arena = torch.zeros(self.plan.n_slots * c.slot_bytes(), dtype=torch.uint8,
                                 device=dev)
        table = wl.block_table(self.plan, c, self.arena.data_ptr())
        self.table = torch.from_numpy(table.view(np.uint8).copy()).to(dev)
        cu = np.concatenate([[0], np.cumsum(self.chunk)]).astype(np.int32)
        self.cu = torch.from_numpy(cu).to(dev)
        self.ctx_d = torch.from_numpy(self.ctx.copy()).to(dev)
        tok_seq = np.repeat(np.arange(c.batch, dtype=np.int32), self.chunk)
        tok_pos = np.concatenate([np.arange(a, a + n, dtype=np.int32)
                                  for a, n in zip(self.ctx, self.chunk)])
        self.tok_seq = torch.from_numpy(tok_seq).to(dev)
        self.tok_pos = torch.from_numpy(tok_pos).to(dev)
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1000003 + 29)
        n = self.n_tok
        self.q = torch.randn((n, c.hq, c.d), generator=g, device=dev).to(torch.bfloat16)
        self.k = torch.randn((n, c.hkv, c.d), generator=g, device=dev).to(torch.bfloat16)
        self.v = torch.randn((n, c.hkv, c.d), generator=g, device=dev).to(torch.bfloat16)
        self.out = torch.zeros((n, c.hq, c.d), dtype=torch.bfloat16, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        # the shared prefix chain: written once through the first hit's table row
        hits = [s for s in range(c.batch) if self.ctx[s] > 0]
        if hits:
            L = int(self.ctx[hits[0]])
            pk = torch.randn((L, c.hkv, c.d), generator=g, device=dev).to(torch.bfloat16)
            pv = torch.randn((L, c.hkv, c.d), generator=g, device=dev).to(torch.bfloat16)
            ts = torch.full((L,), hits[0], dtype=torch.int32, device=dev)
            tp = torch.arange(L, dtype=torch.int32, device=dev)
            rc = self.append_raw(pk, pv, ts, tp, L)
            assert rc == 0, f"prefix append failed: {rc}"
        torch.cuda.synchronize()

    def append_raw(self, k, v, ts, tp, n, stream=None) -> int:
        c = self.cfg
        return self.be.append(k=k.data_ptr(), v=v.data_ptr(), token_seq=ts.data_ptr(),
                              token_pos=tp.data_ptr(), num_tokens=n, num_seqs=c.batch,
                              block_tables=self.table.data_ptr(),
                              max_blocks_per_seq=self.plan.max_blocks, num_kv_heads=c.hkv,
                              head_dim=c.d, block_size=c.block, kv_dtype=c.kv_dtype, layer=0,
                              layer_stride=c.layer_stride(),
                              stream=stream or self.torch.cuda.current_stream().cuda_stream)

    def prefill(self, stream: int, append: int, q=None, k=None, v=None, out=None) -> None:
        c = self.cfg
        rc = self.be.prefill(
            output=out or self.out.data_ptr(), q=q or self.q.data_ptr(),
            k=k or self.k.data_ptr(), v=v or self.v.data_ptr(), cu_seqlens=self.cu.data_ptr(),
            ctx_lens=self.ctx_d.data_ptr(), num_seqs=c.batch, num_tokens=self.n_tok,
            max_chunk=int(self.chunk.max()), num_heads=c.hq, num_kv_heads=c.hkv, head_dim=c.d,
            block_tables=self.table.data_ptr(), max_blocks_per_seq=self.plan.max_blocks,
            block_size=c.block, kv_dtype=c.kv_dtype, layer=0, layer_stride=c.layer_stride(),
            scale=c.scale, append=append, err_word=self.err.data_ptr(), stream=stream)
        if rc != 0:
            raise RuntimeError(f"prefill launch failed: {rc}")

    def append(self, stream: int) -> None:
        rc = self.append_raw(self.k, self.v, self.tok_seq, self.tok_pos, self.n_tok, stream)
        if rc != 0:
            raise RuntimeError(f"append launch failed: {rc}")

    def flops(self) -> int:
        return wl.prefill_flops(self.ctx, self.chunk, self.cfg.hq, self.cfg.d)

    def append_bytes(self) -> int:
        """BF16 K/V read + MX pages written (payload + scales), each once."""
        c = self.cfg
        return self.n_tok * c.hkv * 2 * (c.d * 2 + c.d + c.d // 8)


def prefill_cpu_sample(qq, kk, vv, cfg, step_flops: int, n_tok: int, seconds: float,
                       use_ref: bool) -> dict:
    """The reference CPU attention (kllm_ace_attention, one call per causal
    row, as the reference has no mask) on sampled rows of one prompt and one
    kv head -- qq [n, G, d], kk/vv [n, d] bf16 bits -- scaled to the whole
    step by FLOPs."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    g, n = cfg.group, len(kk)
    rows = list(range(7, n, 16))
    t0 = time.perf_counter()
    flops = reps = 0
    while True:
        for j in rows:
            oracle.attention(qq[j][:, None, :], kk[:j + 1, None], vv[:j + 1, None], 1, cfg.d,
                             j + 1, g, cfg.scale, use_ref=use_ref)
            flops += 4 * cfg.d * g * (j + 1)
        reps += 1
        if time.perf_counter() - t0 > seconds or reps >= 50:
            break
    rate = flops / (time.perf_counter() - t0)
    return {"value": round(n_tok / (step_flops / rate), 2), "unit": "tokens/s", "cores": 1,
            "kind": "reference" if use_ref else "port", "tflops": round(rate / 1e12, 6),
            "sample": f"{len(rows)} causal rows of one {n}-token prompt x {g} heads of one "
                      f"kv head, x {reps} reps; scaled to the step by FLOPs"}


def _use_ref() -> bool:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return oracle.ref() is not None


def run_prefill(args) -> None:
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ["KLLM_GPU_DEVICE"] = str(local)
    import kllm_b200 as kb
    be = kb.Backend()
    if be.backend != kb.KLLM_GPU_CUDA:
        raise RuntimeError("libkllm_gpu: no sm_100 device")
    torch.cuda.set_stream(be.torch_stream())
    cfg = wl.PREFILL_CONFIGS[args.config]
    rig = PrefillRig(cfg, be, torch, local, args.seed)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    for _ in range(args.warmup):
        rig.prefill(sp, append=0)
        rig.append(sp)
    torch.cuda.synchronize()

    # device-timed region: the chunk's Q/K/V/O (940 MB) exceed the 126 MB L2
    clk = Clocks(local)
    clk.start()
    launches0 = be.stats().launches
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3 * args.steps)]
    torch.cuda.synchronize()
    for i in range(args.steps):
        evs[3 * i].record(stream)
        rig.prefill(sp, append=0)
        evs[3 * i + 1].record(stream)
        rig.append(sp)
        evs[3 * i + 2].record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = be.stats().launches - launches0
    t_pf = [evs[3 * i].elapsed_time(evs[3 * i + 1]) for i in range(args.steps)]
    t_ap = [evs[3 * i + 1].elapsed_time(evs[3 * i + 2]) for i in range(args.steps)]
    t_ms = evs[0].elapsed_time(evs[-1])
    assert int(rig.err.item()) == 0, f"prefill error word {int(rig.err.item()):#x}"

    # end to end through the C ABI: pinned host Q/K/V in, O out, one
    # prefill_v2 call with append per step. Two device buffer sets alternate
    # by step, so step s + 1's uploads (their own stream) and step s - 1's
    # read-back (another stream) overlap step s's prefill; events order
    # upload -> prefill -> read-back per buffer set and hold a set until its
    # previous read-back finished
    hq_, hk_, hv_ = (x.cpu().pin_memory() for x in (rig.q, rig.k, rig.v))
    ho = torch.empty_like(rig.out, device="cpu").pin_memory()
    lib, ctx = be.lib, be.ctx
    sets = [tuple(torch.empty_like(x) for x in (rig.q, rig.k, rig.v, rig.out)) for _ in range(2)]
    nbytes = (rig.q.numel() * 2, rig.k.numel() * 2, rig.v.numel() * 2)
    up_s, down_s = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_go, ev_end = torch.cuda.Event(), torch.cuda.Event()
    n_e2e = [0]

    def e2e_step(first=False):
        b = n_e2e[0] & 1
        n_e2e[0] += 1
        dq, dk, dv, do = sets[b]
        if first:                                    # no copy starts before the region opens
            ev_go.record(stream)
            up_s.wait_event(ev_go)
        up_s.wait_event(ev_done[b])                  # the set's previous prefill read it
        for h, d, n in ((hq_, dq, nbytes[0]), (hk_, dk, nbytes[1]), (hv_, dv, nbytes[2])):
            lib.kllm_gpu_memcpy_h2d_async(ctx, d.data_ptr(), h.data_ptr(), n, up_s.cuda_stream)
        ev_in[b].record(up_s)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])                 # the set's previous read-back of O
        rig.prefill(sp, append=1, q=dq.data_ptr(), k=dk.data_ptr(), v=dv.data_ptr(),
                    out=do.data_ptr())
        ev_done[b].record(stream)
        down_s.wait_event(ev_done[b])
        lib.kllm_gpu_memcpy_d2h_async(ctx, ho.data_ptr(), do.data_ptr(), rig.out.numel() * 2,
                                      down_s.cuda_stream)
        ev_out[b].record(down_s)

    def e2e_drain():
        ev_end.record(down_s)
        stream.wait_event(ev_end)                    # every read-back is inside the region

    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_drain()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i == 0)
    e2e_drain()
    e1.record(stream)
    torch.cuda.synchronize()
    if not torch.equal(ho[:2].to(rig.out.device), sets[(n_e2e[0] - 1) & 1][3][:2]):
        raise RuntimeError("end-to-end read-back differs from the device output")
    te_ms = e0.elapsed_time(e1)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        s_last = cfg.batch - 1                    # a full-length prompt
        a0, n0 = int(rig.cu[s_last].item()), int(rig.chunk[s_last])

        def host(x):
            return x[a0:a0 + n0].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        cpu = prefill_cpu_sample(host(rig.q[:, 0:cfg.group]), host(rig.k[:, 0]),
                                 host(rig.v[:, 0]), cfg, rig.flops(), rig.n_tok,
                                 args.cpu_seconds, _use_ref())
    if rank == 0:
        tpeak, tkind = bf16_peak()
        hpeak, hkind = peaks()
        flops = rig.flops()
        pf_ms = float(np.mean(t_pf))
        ap_ms = float(np.mean(t_ap))
        achieved = flops / (pf_ms * 1e-3) / 1e12
        line = {
            "metric": PREFILL_METRIC,
            "value": round(rig.n_tok * args.steps / (t_ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 MMA (tcgen05), fp32 accum; MX-FP8 cached K/V dequantised to bf16",
            "data": "synthetic (seeded torch.randn BF16 Q/K/V ~ N(0,1))",
            "config": {"workload": cfg.name, "prompts": cfg.batch, "prompt_len": cfg.ctx_lo,
                       "shared_prefix_hits": int((rig.ctx > 0).sum()),
                       "shared_prefix_tokens": int(rig.ctx.max()), "new_tokens": rig.n_tok,
                       "hq": cfg.hq, "hkv": cfg.hkv, "head_dim": cfg.d, "block": cfg.block,
                       "kv_format": "mx-fp8-e4m3 (e4m3 scale per 8)",
                       "l2": "inputs larger than L2 (chunk Q/K/V/O 940 MB per step)"},
            "attention_tflops": round(achieved, 2),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": tpeak,
                         "unit": "TFLOP/s", "frac": round(achieved / tpeak, 4),
                         "peak_kind": tkind, "traffic": None,
                         "kernel": "prefill_kernel<4> (tcgen05, causal algorithmic FLOPs)",
                         "launch_ms": round(pf_ms, 4)},
            "append_roofline": {"bound": "hbm",
                                "achieved": round(rig.append_bytes() / (ap_ms * 1e-3) / 1e9, 1),
                                "peak": hpeak, "unit": "GB/s", "peak_kind": hkind,
                                "frac": round(rig.append_bytes() / (ap_ms * 1e-3) / 1e9 / hpeak,
                                              4),
                                "kernel": "append_warp_kernel<128> (MX-FP8 quantize-on-write)", "launch_ms": round(ap_ms, 4)},
            "e2e": {"value": round(rig.n_tok * args.steps / (te_ms * 1e-3), 1),
                    "unit": "tokens/s",
                    "h2d_bytes_per_step": int(sum(nbytes)),
                    "d2h_bytes_per_step": int(rig.out.numel() * 2)},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    be.close()


def run_reference_prefill(args) -> None:
    """The reference CPU attention on the C5 sample (host arrays only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cfg = wl.PREFILL_CONFIGS[args.config]
    ctx, chunk = wl.prefill_split(cfg)
    n_tok = int(chunk.sum())
    n = int(chunk[-1])                            # a full-length prompt
    q = wl.normal_bf16(args.seed, wl.ST_PQ, 0, (n, cfg.hq, cfg.d))[:, :cfg.group]
    k = wl.normal_bf16(args.seed, wl.ST_PK, 0, (n, cfg.hkv, cfg.d))[:, 0]
    v = wl.normal_bf16(args.seed, wl.ST_PV, 0, (n, cfg.hkv, cfg.d))[:, 0]
    flops = wl.prefill_flops(ctx, chunk, cfg.hq, cfg.d)
    use_ref = _use_ref()
    per = args.cpu_seconds / max(1, args.steps)
    for _ in range(min(args.warmup, 1)):
        prefill_cpu_sample(q, k, v, cfg, flops, n_tok, 0.0, use_ref)
    samples = [prefill_cpu_sample(q, k, v, cfg, flops, n_tok, per, use_ref)
               for _ in range(args.steps)]
    value = float(np.mean([x["value"] for x in samples]))
    line = {
        "impl": "reference", "metric": PREFILL_METRIC, "value": round(value, 2),
        "unit": "tokens/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * n_tok / value, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 products, fp32 accum (CPU)",
        "data": "synthetic",
        "config": {"workload": cfg.name, "prompts": cfg.batch, "prompt_len": cfg.ctx_lo},
        "cpu_baseline": dict(samples[-1], value=round(value, 2)),
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# reference arm (CPU)
# ---------------------------------------------------------------------------

TABLE_METRIC = ("content-addressed block-table build (SHA-256 block key + index probe + "
                "24-byte entry): table blocks/s")


def chained_keys(tokens: np.ndarray, lens: np.ndarray, starts: np.ndarray, block: int):
    """Host block keys with hashlib, one running hash per sequence (the same
    values as hashing every prefix from scratch)."""
    import hashlib
    keys = []
    for s, n in enumerate(lens.tolist()):
        h = hashlib.sha256()
        seq = tokens[starts[s]:starts[s] + n]
        row = []
        for b in range((n + block - 1) // block):
            h.update(seq[b * block:(b + 1) * block].tobytes())
            row.append(h.copy().digest())
        keys.append(row)
    return keys


class TableRig:
    """A table-build workload resident on the GPU: token ids, the index mirror
    (warm: every block indexed; prefix: the shared prefix chain only), the
    table, keys, workspace and miss list."""

    def __init__(self, tcfg, be, torch, device: int, seed: int = 0):
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import tablecase as tc
        self.tcfg, self.be, self.torch = tcfg, be, torch
        c = tcfg.lengths
        self.block = c.block
        self.tokens, self.starts, self.lens = wl.table_tokens(tcfg, seed)
        S = len(self.lens)
        nb = (self.lens + self.block - 1) // self.block
        self.blocks = int(nb.sum())
        self.max_blocks = int(nb.max())
        if tcfg.warm == "prefix":
            ctx, chunk = wl.prefill_split(c)
            self.plan = wl.plan_prefill_pages(c, ctx, chunk, seed)
            indexed = [(s, b) for s in range(S) if ctx[s] for b in range(int(ctx[s]) // c.block)]
        else:
            self.plan = wl.plan_pages(c, self.lens, seed)
            indexed = [(s, b) for s in range(S) for b in range(int(nb[s]))]
        keys = chained_keys(self.tokens, self.lens, self.starts, self.block)
        self.entries = tc.empty_index(tcfg.index_capacity)
        seen = set()
        for s, b in indexed:
            k = keys[s][b]
            if k not in seen:
                seen.add(k)
                tc.index_insert(self.entries, k, int(self.plan.slots[s, b]))
        self.expected_hits = len(indexed)
        self.base = 0x7f0000000000
        self.slot_bytes = c.slot_bytes()
        self.want_table = wl.block_table(self.plan, c, self.base)
        if tcfg.warm == "prefix":
            hit = np.zeros(self.plan.slots.shape, bool)
            for s, b in indexed:
                hit[s, b] = True
            self.want_table[~hit] = 0
        dev = torch.device("cuda", device)
        self.d_tokens = torch.from_numpy(self.tokens.view(np.int32)).to(dev)
        self.d_starts = torch.from_numpy(self.starts).to(dev)
        self.d_lens = torch.from_numpy(self.lens).to(dev)
        self.d_index = torch.from_numpy(self.entries.view(np.uint8).copy()).to(dev)
        self.table = torch.zeros(S * self.max_blocks * 24, dtype=torch.uint8, device=dev)
        self.hashes = torch.zeros(S * self.max_blocks * 32, dtype=torch.uint8, device=dev)
        self.ws_bytes = be.lib.kllm_gpu_table_workspace_size(S, self.max_blocks, self.block)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.miss_list = torch.zeros(2 * self.blocks, dtype=torch.int32, device=dev)
        self.miss_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.hit_miss = torch.zeros(2, dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    def build(self, stream: int, tokens=None, starts=None, lens=None) -> None:
        rc = self.be.build_tables(
            token_ids=tokens or self.d_tokens.data_ptr(),
            token_starts=starts or self.d_starts.data_ptr(),
            seq_lens=lens or self.d_lens.data_ptr(), first_block=None,
            num_seqs=len(self.lens), max_blocks_per_seq=self.max_blocks, block_size=self.block,
            index=self.d_index.data_ptr(), index_capacity=self.tcfg.index_capacity, now_ns=0,
            arena_base=self.base, slot_bytes=self.slot_bytes, total_slots=self.plan.n_slots,
            k_offset=0, v_offset=self.tcfg.lengths.page_bytes(),
            block_tables=self.table.data_ptr(), hashes=self.hashes.data_ptr(),
            workspace=self.ws.data_ptr(), workspace_bytes=self.ws_bytes,
            miss_list=self.miss_list.data_ptr(), miss_capacity=self.blocks,
            miss_count=self.miss_count.data_ptr(), hit_miss=self.hit_miss.data_ptr(),
            err_word=self.err.data_ptr(), stream=stream)
        if rc != 0:
            raise RuntimeError(f"block-table build failed: {rc}")

    def check(self) -> None:
        """The table equals the planned one (warm: every block; prefix: the
        shared chain), the miss count is the unindexed blocks."""
        self.torch.cuda.synchronize()
        got = self.table.cpu().numpy().view(wl.ENTRY_DTYPE).reshape(self.want_table.shape)
        assert (got == self.want_table).all(), "block-table build differs from the plan"
        assert int(self.miss_count.item()) == self.blocks - self.expected_hits
        assert int(self.err.item()) == 0

    def algorithmic_bytes(self) -> int:
        """Token ids read once, one index entry (48 B) per block, table and
        keys written ([S][max_blocks]), midstates written and read once."""
        S = len(self.lens)
        msg_blocks = int((self.lens // 16).sum())
        return (4 * int(self.lens.sum()) + 48 * self.blocks +
                (24 + 32) * S * self.max_blocks + 64 * msg_blocks + 12 * S)


def run_tables(args) -> None:
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(local)
    os.environ["KLLM_GPU_DEVICE"] = str(local)
    import kllm_b200 as kb
    be = kb.Backend()
    if be.backend != kb.KLLM_GPU_CUDA:
        raise RuntimeError("libkllm_gpu: no sm_100 device")
    torch.cuda.set_stream(be.torch_stream())
    tcfg = wl.TABLE_CONFIGS[args.config]
    rig = TableRig(tcfg, be, torch, local, args.seed)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    for _ in range(args.warmup):
        rig.build(sp)
    rig.check()
    # the workload (~25-60 MB) fits in L2: every timed build follows a
    # 256 MB write that flushes it
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
    clk = Clocks(local)
    clk.start()
    launches0 = be.stats().launches
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        evs[2 * i].record(stream)
        rig.build(sp)
        evs[2 * i + 1].record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = be.stats().launches - launches0
    times = [evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(args.steps)]
    t_ms = float(sum(times))

    # end to end through the C ABI: pinned host token ids / starts / lengths
    # in, the build, the miss count and hit/miss counters back
    h_tok = torch.from_numpy(rig.tokens.view(np.int32)).pin_memory()
    h_st = torch.from_numpy(rig.starts).pin_memory()
    h_ln = torch.from_numpy(rig.lens).pin_memory()
    h_out = torch.zeros(6, dtype=torch.int32).pin_memory()
    d_tok, d_st, d_ln = (torch.empty_like(x, device=f"cuda:{local}") for x in (h_tok, h_st, h_ln))
    lib, ctx = be.lib, be.ctx
    h2d = [(d_tok, h_tok, rig.tokens.nbytes), (d_st, h_st, rig.starts.nbytes),
           (d_ln, h_ln, rig.lens.nbytes)]

    def e2e_step():
        for d, h, n in h2d:
            lib.kllm_gpu_memcpy_h2d_async(ctx, d.data_ptr(), h.data_ptr(), n, sp)
        rig.build(sp, d_tok.data_ptr(), d_st.data_ptr(), d_ln.data_ptr())
        lib.kllm_gpu_memcpy_d2h_async(ctx, h_out.data_ptr(), rig.miss_count.data_ptr(), 4, sp)
        lib.kllm_gpu_memcpy_d2h_async(ctx, h_out[2:].data_ptr(), rig.hit_miss.data_ptr(), 16, sp)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    e_ms = 0.0
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms += e0.elapsed_time(e1)
    assert int(h_out[0]) == rig.blocks - rig.expected_hits

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = table_cpu_sample(rig, args.cpu_seconds)
    if rank == 0:
        hpeak, hkind = peaks()
        per_ms = t_ms / args.steps
        gbs = rig.algorithmic_bytes() / (per_ms * 1e-3) / 1e9
        longest = int(rig.lens.max()) // 16
        line = {
            "metric": TABLE_METRIC,
            "value": round(rig.blocks * args.steps / (t_ms * 1e-3), 1), "unit": "blocks/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32",
            "data": "synthetic (seeded token ids in [0, 128256))",
            "config": {"workload": tcfg.name, "requests": len(rig.lens),
                       "tokens": int(rig.lens.sum()), "table_blocks": rig.blocks,
                       "block": rig.block, "index_capacity": tcfg.index_capacity,
                       "indexed_blocks": rig.expected_hits,
                       "l2": "flushed before every timed build (256 MB write)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hpeak,
                         "unit": "GB/s", "frac": round(gbs / hpeak, 5), "peak_kind": hkind,
                         "traffic": None,
                         "kernel": "chain_kernel + finalize_kernel (one build)",
                         "note": "latency-bound: the SHA-256 chain of a sequence is "
                                 "sequential; the longest request has "
                                 f"{longest} 64-byte message blocks",
                         "chain_message_blocks_longest": longest},
            "e2e": {"value": round(rig.blocks * args.steps / (e_ms * 1e-3), 1),
                    "unit": "blocks/s",
                    "h2d_bytes_per_step": int(sum(n for _, _, n in h2d)),
                    "d2h_bytes_per_step": 20},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    be.close()


class RefTables:
    """The reference's path on a table workload: its own index (cache_index.c)
    holding the same keys, OpenSSL SHA256 of every block's prefix spread over
    host threads, then kllm_index_lookup per block on one thread."""

    def __init__(self, tcfg, seed: int, nthreads: int):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        self.ok = oracle.ref_index_lib() is not None
        self.tokens, self.starts, self.lens = wl.table_tokens(tcfg, seed)
        c = tcfg.lengths
        self.block, self.nthreads = c.block, nthreads
        nb = (self.lens + c.block - 1) // c.block
        self.blocks, self.max_blocks = int(nb.sum()), int(nb.max())
        if not self.ok:
            return
        keys = chained_keys(self.tokens, self.lens, self.starts, c.block)
        if tcfg.warm == "prefix":
            ctx, _ = wl.prefill_split(c)
            indexed = {keys[s][b] for s in range(len(self.lens)) if ctx[s]
                       for b in range(int(ctx[s]) // c.block)}
        else:
            indexed = {k for row in keys for k in row}
        self.expected_hits = sum(1 for row in keys for k in row if k in indexed)
        self.idx = oracle.RefIndex(tcfg.index_capacity, 1 << 22)
        for k in sorted(indexed):
            self.idx.insert(k)

    def run(self):
        """(key seconds, lookup seconds) of one build; checks the hit count."""
        slots, _, tk, tl = self.idx.build_slots_mt(self.tokens, self.starts, self.lens,
                                                   self.max_blocks, self.block, self.nthreads)
        assert int((slots >= 0).sum()) == self.expected_hits
        return tk, tl


def table_cpu_sample(rig, seconds: float) -> dict | None:
    n = os.cpu_count() or 1
    ref = RefTables(rig.tcfg, 0, n)
    if not ref.ok:
        return None
    t0 = time.perf_counter()
    reps, tk, tl = 0, 0.0, 0.0
    while reps < 200:
        a, b = ref.run()
        reps, tk, tl = reps + 1, tk + a, tl + b
        if time.perf_counter() - t0 > min(seconds, 10.0):
            break
    per = (tk + tl) / reps
    return {"value": round(ref.blocks / per, 1), "unit": "blocks/s", "cores": n,
            "kind": "reference", "key_seconds": round(tk / reps, 6),
            "lookup_seconds": round(tl / reps, 6),
            "sample": f"the whole workload x {reps} reps: OpenSSL SHA256 of every "
                      f"block's prefix over {n} threads, then kllm_index_lookup on one"}


def run_reference_tables(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    tcfg = wl.TABLE_CONFIGS[args.config]
    n = os.cpu_count() or 1
    ref = RefTables(tcfg, args.seed, n)
    if not ref.ok:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libkllm_ref_index.so was not built here"}), flush=True)
        return
    for _ in range(args.warmup):
        ref.run()
    t = sum(sum(ref.run()) for _ in range(args.steps))
    value = ref.blocks * args.steps / t
    line = {
        "impl": "reference", "metric": TABLE_METRIC, "value": round(value, 1),
        "unit": "blocks/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
        "config": {"workload": tcfg.name, "block": tcfg.lengths.block,
                   "index_capacity": tcfg.index_capacity},
        "cpu_baseline": {"value": round(value, 1), "unit": "blocks/s", "cores": n,
                         "kind": "reference",
                         "sample": "the whole workload per step: OpenSSL SHA256 of every "
                                   f"block's prefix over {n} threads, then kllm_index_lookup"},
        "e2e": {"value": round(value, 1), "unit": "blocks/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


LM_HEAD_METRIC = "lm_head projection + token sampling: tokens/s (rows sampled per second)"


def run_lm_head(args) -> None:
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(local)
    os.environ["KLLM_GPU_DEVICE"] = str(local)
    import kllm_b200 as kb
    be = kb.Backend()
    if be.backend != kb.KLLM_GPU_CUDA:
        raise RuntimeError("libkllm_gpu: no sm_100 device")
    torch.cuda.set_stream(be.torch_stream())
    c = wl.LM_HEAD_CONFIGS[args.config]
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed * 1000003 + 41)
    R, H, V = c.rows, c.hidden, c.vocab
    hid = torch.randn((R, H), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((V, H), generator=g, device=dev) * (1.5 / math.sqrt(H))).to(torch.bfloat16)
    logits = torch.empty((R, V), dtype=torch.float32, device=dev)
    tok = torch.empty(R, dtype=torch.int32, device=dev)
    ws_b = be.lib.kllm_gpu_lm_head_workspace_size(R, V)
    ws = torch.empty(ws_b, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rng = np.random.default_rng(args.seed)
    if c.sampling == "greedy":
        meth = temp = topk = None
    else:
        meth = torch.from_numpy(rng.choice([0, 1, 2, 3], R).astype(np.int32)).to(dev)
        temp = torch.from_numpy(rng.choice([0.7, 1.0], R).astype(np.float32)).to(dev)
        topk = torch.from_numpy(rng.choice([40, 50, 200], R).astype(np.int32)).to(dev)
    uni = torch.from_numpy(rng.random(R).astype(np.float32)).to(dev)
    st = torch.cuda.current_stream()
    sp = st.cuda_stream

    def step(hptr=None, tptr=None):
        rc = be.lm_head(hidden=hptr or hid.data_ptr(), weight=w.data_ptr(), num_rows=R,
                        hidden_dim=H, vocab=V, logits=logits.data_ptr(),
                        method=meth.data_ptr() if meth is not None else None,
                        temperature=temp.data_ptr() if temp is not None else None,
                        top_k=topk.data_ptr() if topk is not None else None,
                        uniform=uni.data_ptr(), tokens=tptr or tok.data_ptr(),
                        workspace=ws.data_ptr(),
                        workspace_bytes=ws_b, err_word=err.data_ptr(), stream=sp)
        if rc != 0:
            raise RuntimeError(f"lm_head failed: {rc}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # a spot check of the tokens against the logits the kernel wrote
    lg0 = logits[0].cpu().numpy()
    if c.sampling == "greedy":
        assert int(tok[0].item()) == int(np.argmax(lg0)), "greedy token is not the argmax"
    assert int(err.item()) == 0
    clk = Clocks(local)
    clk.start()
    launches0 = be.stats().launches
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step()          # weights 1.05 GB per step: every step streams past the 126 MB L2
    e1.record(st)
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = be.stats().launches - launches0
    t_ms = e0.elapsed_time(e1)
    # end to end through the C ABI: pinned hidden states in, tokens out; two
    # hidden-state buffers alternate by step so the next step's upload (its
    # own stream) overlaps this step's projection, ordered by events
    h_h = hid.cpu().pin_memory()
    h_t = torch.empty(R, dtype=torch.int32).pin_memory()
    d_hs = [torch.empty_like(hid) for _ in range(2)]
    d_ts = [torch.empty_like(tok) for _ in range(2)]
    lib, ctx = be.lib, be.ctx
    up_s, down_s = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_tok = [torch.cuda.Event() for _ in range(2)]
    ev_go, ev_end = torch.cuda.Event(), torch.cuda.Event()
    n_e2e = [0]

    def e2e_step(first=False):
        b = n_e2e[0] & 1
        n_e2e[0] += 1
        if first:                                    # no copy starts before the region opens
            ev_go.record(st)
            up_s.wait_event(ev_go)
        up_s.wait_event(ev_done[b])                  # the buffer's previous projection read it
        lib.kllm_gpu_memcpy_h2d_async(ctx, d_hs[b].data_ptr(), h_h.data_ptr(), R * H * 2,
                                      up_s.cuda_stream)
        ev_in[b].record(up_s)
        st.wait_event(ev_in[b])
        st.wait_event(ev_tok[b])                     # the buffer's previous tokens were read
        step(d_hs[b].data_ptr(), d_ts[b].data_ptr())
        ev_done[b].record(st)
        down_s.wait_event(ev_done[b])
        lib.kllm_gpu_memcpy_d2h_async(ctx, h_t.data_ptr(), d_ts[b].data_ptr(), R * 4,
                                      down_s.cuda_stream)
        ev_tok[b].record(down_s)

    def e2e_drain():
        ev_end.record(down_s)
        st.wait_event(ev_end)

    for _ in range(args.warmup):
        e2e_step()
    e2e_drain()
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(args.steps):
        e2e_step(i == 0)
    e2e_drain()
    e1.record(st)
    torch.cuda.synchronize()
    te_ms = e0.elapsed_time(e1)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = lm_head_cpu_sample(hid, w, R, V, args.cpu_seconds)
    if rank == 0:
        per = t_ms / args.steps
        flops = 2.0 * R * H * V
        nbytes = V * H * 2 + R * H * 2 + R * V * 4
        hpeak, hkind = peaks()
        tpeak, tkind = bf16_peak()
        gbs = nbytes / (per * 1e-3) / 1e9
        line = {
            "metric": LM_HEAD_METRIC, "value": round(R * args.steps / (t_ms * 1e-3), 1),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 MMA (tcgen05), fp32 accum",
            "data": "synthetic (seeded torch.randn hidden states and weights)",
            "config": {"workload": c.name, "rows": R, "hidden": H, "vocab": V,
                       "sampling": c.sampling,
                       "l2": "weights 1.05 GB per step, larger than L2"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hpeak, "unit": "GB/s",
                         "frac": round(gbs / hpeak, 4), "peak_kind": hkind, "traffic": None,
                         "kernel": "lm_head_kernel<2> + sample_kernel (one step)",
                         "algorithmic_bytes": nbytes},
            "tensor": {"achieved_tflops": round(flops / (per * 1e-3) / 1e12, 1),
                       "peak": tpeak, "frac": round(flops / (per * 1e-3) / 1e12 / tpeak, 4)},
            "e2e": {"value": round(R * args.steps / (te_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": R * H * 2, "d2h_bytes_per_step": R * 4},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    be.close()


def lm_head_cpu_sample(hid, w, R, V, seconds):
    """The projection of one row against the whole vocabulary by the oracle
    port (the reference has no lm_head: its GPU path returns zero logits),
    then the reference's own greedy sampler (decode_loop.c:58-70) over those
    logits, scaled to the batch."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    h = hid[:1].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
    wt = w.contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
    t0 = time.perf_counter()
    lg = oracle.lm_head_logits(h, wt)[0]
    t_proj = time.perf_counter() - t0
    t0 = time.perf_counter()
    if oracle.ref_sampling_lib() is not None:
        oracle.ref_sampling_lib().ref_sample_token(oracle.ptr(lg), V, 0, 0.0, 0, 0.0)
        kind = "port (projection) + reference (sampler)"
    else:
        oracle.sample_token(lg, 0, 0.0, 0, 0.0)
        kind = "port"
    t_samp = time.perf_counter() - t0
    per_row = t_proj + t_samp
    return {"value": round(1.0 / per_row, 3), "unit": "tokens/s", "cores": 1, "kind": "port",
            "detail": kind, "projection_s_per_row": round(t_proj, 4),
            "sampling_s_per_row": round(t_samp, 6),
            "sample": f"one row x {V} vocabulary rows x {hid.shape[1]} (fp32 sums), then "
                      "greedy sampling; per row, so tokens/s for the batch is the same"}


def torch_int16():
    import torch
    return torch.int16


ARRIVAL_METRIC = "KV block arrival into VRAM by content key (wavefront submit -> poll): GB/s"


def run_arrival(args) -> None:
    """Store file of random block records in a temporary directory (page
    cache resident: this measures the host-staged path, not a drive), an
    index of their keys, then per step 64 wavefronts of 64 blocks each
    submitted and polled to completion; wall time on the host from the first
    submit to the last completion (the completions are observed by polling)."""
    import ctypes
    import tempfile
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(local)
    import kllm_b200 as kb
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tablecase as tc
    acfg = wl.ARRIVAL_CONFIGS[args.config]
    lib = kb.load()
    rng = np.random.default_rng(args.seed)
    n, rb = acfg.blocks, acfg.record_bytes
    data = rng.integers(0, 256, (n, rb), dtype=np.uint8)
    keys = [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(n)]
    entries = tc.empty_index(1 << (2 * n - 1).bit_length())
    for r in range(n):
        tc.index_insert(entries, keys[r], r)
    dev = torch.zeros(n * rb, dtype=torch.uint8, device=f"cuda:{local}")
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "kv_store.bin")
        with open(path, "wb") as f:
            f.write(data.tobytes())
        ctx = lib.kllm_wavefront_create2(path.encode(), local, rb, acfg.staging)
        if not ctx:
            raise RuntimeError("kllm_wavefront_create2 failed")
        try:
            assert lib.kllm_wavefront_set_index(ctx, entries.ctypes.data, len(entries), rb,
                                                0) == 0
            perm = rng.permutation(n)
            wfs = []
            for w in range(0, n, 64):
                wf = kb.Wavefront()
                wf.num_blocks, wf.flags, wf.sequence_id = 64, 2, w
                for i in range(64):
                    r = int(perm[w + i])
                    ctypes.memmove(wf.blocks[i].obj_key, keys[r], 32)
                    wf.blocks[i].vram_dest_addr = dev.data_ptr() + (w + i) * rb
                    wf.blocks[i].block_size = rb
                wfs.append(wf)
            comp = (kb.WfCompletion * 64)()

            def one_step():
                for wf in wfs:
                    if lib.kllm_wavefront_submit(ctx, ctypes.byref(wf)) != 0:
                        raise RuntimeError("kllm_wavefront_submit refused")
                done = failed = 0
                while done < len(wfs):
                    k = lib.kllm_wavefront_wait(ctx, comp, 64, 10000)
                    if k <= 0:
                        raise RuntimeError("no wavefront completion within 10 s")
                    done += k
                    failed += sum(comp[i].blocks_failed for i in range(k))
                return failed

            for _ in range(args.warmup):
                assert one_step() == 0
            torch.cuda.synchronize()
            host = dev.cpu().numpy().reshape(n, rb)
            assert np.array_equal(host, data[perm]), "arrived blocks differ from the store"
            t0 = time.perf_counter()
            for _ in range(args.steps):
                one_step()
            t = time.perf_counter() - t0
            assert lib.kllm_wavefront_error(ctx) == 0
        finally:
            lib.kllm_wavefront_destroy(ctx)
    # the ceiling of a host-staged path: one large page-locked host-to-device copy
    pin = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dst = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = 0.0
    for _ in range(4):
        e0.record()
        dst.copy_(pin, non_blocking=True)
        e1.record()
        e1.synchronize()
        h2d = max(h2d, pin.numel() / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    del pin, dst
    # I/O threads and scatter launches, as the wavefront context arranges them
    nthr = min(4, acfg.staging // 2)
    chunk = max(2 << 20, (rb + 15) // 16 * 16)
    per_thread = -(-64 // nthr)
    per_chunk = chunk // ((rb + 15) // 16 * 16)
    launches = args.steps * (n // 64) * nthr * -(-per_thread // per_chunk)
    if rank == 0:
        gbs = n * rb * args.steps / t / 1e9
        line = {
            "metric": ARRIVAL_METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded random block records in a page-cached store file)",
            "config": {"workload": acfg.name, "blocks": n, "record_bytes": rb,
                       "wavefronts_per_step": n // 64, "staging_buffers": acfg.staging,
                       "io_threads": nthr,
                       "source": "page cache (host-staged path; no NVMe drive measured)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 3), "peak": peaks()[0],
                         "unit": "GB/s", "frac": round(gbs / peaks()[0], 5),
                         "peak_kind": peaks()[1], "traffic": None,
                         "h2d_copy_gbs": round(h2d, 2), "frac_of_h2d_copy": round(gbs / h2d, 4),
                         "note": "host-side path: pread into page-locked chunks, one "
                                 "host-to-device copy and one scatter launch per chunk; the "
                                 "bound is the host-to-device link (h2d_copy_gbs, one 256 MiB "
                                 "page-locked copy measured here), not HBM"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": n * rb,
                    "d2h_bytes_per_step": 0},
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle
    import kvcase
    lib = oracle.ref()
    kind, prefix = ("reference", "ref") if lib is not None else ("port", "orc")
    if lib is None:
        lib = oracle.orc()
    cfg = wl.CONFIGS[args.config]
    lens_all = wl.context_lengths(cfg, args.seed)
    order = np.argsort(lens_all)
    pick = sorted(int(i) for i in order[np.linspace(0, len(order) - 1, 24).astype(int)])
    hc = kvcase.build_case(cfg, seq_lens=lens_all[pick], layers=1, tail_fill=0)
    c = hc.cfg
    nthreads = os.cpu_count() or 1
    table = hc.host_table()
    sample_bytes = wl.algorithmic_bytes(c, hc.seq_lens, layers=1)

    def step():
        return oracle.harness_decode(lib, prefix, hc.q[0], table, hc.seq_lens, c.hq, c.hkv,
                                     c.d, hc.plan.max_blocks, c.scale, c.block, c.kv_dtype, 0,
                                     nthreads)[1]
    for _ in range(args.warmup):
        step()
    walls = [step() for _ in range(args.steps)]
    t = sum(walls)
    value = sample_bytes * args.steps / t / 1e9
    full_step_s = (t / args.steps) * wl.algorithmic_bytes(cfg, lens_all) / sample_bytes
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 products, fp32 accum (CPU; MX-FP8 KV dequantised to bf16 exactly)",
        "data": "synthetic",
        "config": {"workload": cfg.name, "batch": cfg.batch, "layers": cfg.layers,
                   "hq": cfg.hq, "hkv": cfg.hkv, "head_dim": cfg.d, "block": cfg.block,
                   "kv_format": "mx-fp8-e4m3 (e4m3 scale per 8)"},
        "tokens_per_s": round(cfg.batch / full_step_s, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nthreads,
                         "kind": kind,
                         "sample": f"layer 0 of {len(pick)} requests spanning the context "
                                   f"range ({int(hc.seq_lens.sum())} tokens, "
                                   f"{sample_bytes / 1e6:.1f} MB) per step"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kllm", choices=["kllm", "reference"])
    ap.add_argument("--config", default=wl.C3.name,
                    choices=list(wl.CONFIGS) + list(wl.PREFILL_CONFIGS) +
                    list(wl.TABLE_CONFIGS) + list(wl.ARRIVAL_CONFIGS) +
                    list(wl.LM_HEAD_CONFIGS))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--merge", default="p2p", choices=["p2p", "nccl"],
                    help="split-KV exchange at N > 1 (one long context): peer-memory kernel "
                         "or NCCL all-gather + merge kernel")
    ap.add_argument("--arena-layout", default="layer-major",
                    choices=["layer-major", "slot-major"],
                    help="layer-major: each layer's pages form one region (layer_stride = "
                         "n_slots x 2 pages); slot-major: a slot holds all layers of a block")
    ap.add_argument("--per-request-compare", action="store_true",
                    help="also time the decode step issued one request per launch (the "
                         "reference scheduler's loop), reported beside the batched step")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch each layer's decode only after the previous kernel completed "
                         "(no KLLM_DECODE_OVERLAP_PREV)")
    ap.add_argument("--shard-of", default=None, metavar="R/N",
                    help="decode only the requests rank R of an N-way split would own, on "
                         "one GPU (per-GPU behaviour of an N-GPU run)")
    ap.add_argument("--decode-entry", default="context", choices=["context", "noalloc"],
                    help="decode through kllm_gpu_paged_attention_v2 (context workspace) or "
                         "kllm_gpu_paged_attention_v2_noalloc (fixed in-library scratch)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (smaller captures for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    prefill = args.config in wl.PREFILL_CONFIGS
    if args.config in wl.TABLE_CONFIGS:
        (run_reference_tables if args.impl == "reference" else run_tables)(args)
        return
    if args.config in wl.LM_HEAD_CONFIGS:
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "the reference has no lm_head: its GPU inference returns an "
                                  "all-zero logit vector and takes its argmax "
                                  "(userspace/compute/infer_gpu.c:212-229)"}), flush=True)
            return
        run_lm_head(args)
        return
    if args.config in wl.ARRIVAL_CONFIGS:
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "the reference's kllm_wavefront_submit/poll are stubs "
                                  "(userspace/gpu/nvme_ep_wavefront.c:74-104): nothing is "
                                  "read and no completion is ever reported"}), flush=True)
            return
        run_arrival(args)
        return
    if args.impl == "reference":
        (run_reference_prefill if prefill else run_reference)(args)
    else:
        (run_prefill if prefill else run_kllm)(args)


if __name__ == "__main__":
    main()
