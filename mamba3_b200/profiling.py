"""Instrumentation hooks: per-stage CUDA events inside the layer forward, clock sampling."""

from __future__ import annotations

import contextlib
import statistics
import threading
import time

_tls = threading.local()


def current_stage_events():
    return getattr(_tls, "events", None)


@contextlib.contextmanager
def stage_events(events):
    """Record ``events`` (len = stages + 1) around the stages of the next layer forward on this thread."""
    prev = getattr(_tls, "events", None)
    _tls.events = events
    try:
        yield
    finally:
        _tls.events = prev


# NVML clock-event reason bits
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clocks"}


class ClockSampler:
    """Samples SM clock, power and clock-event reasons of one GPU every `period` seconds (NVML),
    fine enough to put several samples inside a timed region of a few tens of milliseconds."""

    def __init__(self, torch_device_index: int, period: float = 0.005):
        import torch

        self.period = period
        self.samples = []
        self._stop = threading.Event()
        self._thr = None
        self.handle = None
        self.err = None
        try:
            import pynvml

            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(torch_device_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            self.nv = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 -- reported in the JSON, not fatal
            self.err = f"{type(e).__name__}: {e}"

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                pw = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((time.time(), sm, rs, pw))
            except Exception as e:  # noqa: BLE001
                self.err = f"{type(e).__name__}: {e}"
            self._stop.wait(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self):
        if self.handle is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.err}
        sms = [s[1] for s in self.samples]
        bits = 0
        for s in self.samples:
            bits |= int(s[2])
        reasons = sorted(n for b, n in _REASONS.items() if bits & b and n != "gpu_idle")
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": self.max_sm, "reasons": reasons,
                "samples": len(sms), "power_w_max": round(max(s[3] for s in self.samples), 1)}


def train_step_profile(batch: int = 16, seqlen: int = 4096, rows: int = 24) -> str:
    """Per-kernel device time of one config-1 KulaMamba training step (forward + backward,
    bf16, random init, synthetic input) from torch's profiler, after three warm-up steps.  For
    reading where the time goes; the bench's training-step figure is timed without a profiler."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from .mamba3 import KulaMamba

    torch.manual_seed(0)
    layer = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).train()
    x = torch.randn(batch, seqlen, 768, device="cuda").to(torch.bfloat16)

    def step():
        layer.zero_grad(set_to_none=True)
        layer(x).float().sum().backward()

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    return prof.key_averages().table(sort_by="self_cuda_time_total", row_limit=rows, max_name_column_width=72)


def kernel_workload(case: str, reps: int = 3) -> None:
    """Small fixed workloads for per-kernel captures (ncu -k <kernel> -s <warm-up launches>):
    each runs its kernels once as warm-up and then `reps` times.

    cfg3     layer forward, d_model 2048 / 64 heads / mimo_rank 4, bf16, x (2, 8192, 2048): the
             fused kernel at R = 4 (prep_kernel, ssd_fused_kernel per forward)
    chunked  chunked_ssd on pre-processed bf16 tensors (2, 4096) x 24 heads, P 64, N 128, R 2,
             trapezoid: gen_state_kernel, the scan, gen_out_kernel
    chunked_bwd  its backward on the same tensors (tensor-core path): the chunk-state kernels, the
             two scans, bwd_out_kernel, the sums and the suffix pass
    step     one layer's decode step at config-4 shapes (batch 256 x 24 heads, compact state):
             step_prep_kernel, step_stream_kernel
    fp32     config-0 layer forward (4, 1024, 768) fp32: prep, angle prefix, the tf32
             chunk_state_kernel, the scan, the tf32 chunk_out_kernel
    in_proj  the config-1 input projection with its B / C 1/rms epilogue: x (16 x 4096, 768) bf16
             -> proj (65536, 3696) (in_proj_kernel)
    decode   config-4 decoding: the 24-layer LM, batch 256, a 16-token prompt, then `reps` token
             steps of the CUDA-graph decoder (every kernel of a token step, in graph order)"""
    import torch

    from . import ops
    from .mamba3 import KulaMamba
    from .ssd import chunked_ssd

    g = torch.Generator(device="cuda").manual_seed(11)
    torch.manual_seed(0)
    with torch.no_grad():
        if case == "cfg3":
            m = KulaMamba(d_model=2048, d_state=128, headdim=64, mimo_rank=4).cuda().to(torch.bfloat16).eval()
            x = torch.randn(2, 8192, 2048, device="cuda", generator=g).to(torch.bfloat16)
            run = lambda: m(x)  # noqa: E731
        elif case == "fp32":
            m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().eval()
            x = torch.randn(4, 1024, 768, device="cuda", generator=g)
            run = lambda: m(x)  # noqa: E731
        elif case == "chunked":
            B, T, H, P, N, R = 2, 4096, 24, 64, 128, 2
            r = lambda *sh: torch.randn(*sh, device="cuda", generator=g).to(torch.bfloat16)  # noqa: E731
            args = (r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R),
                    torch.rand(B, T, H, device="cuda", generator=g) * 0.1, -torch.rand(H, device="cuda", generator=g),
                    torch.randn(H, device="cuda", generator=g), r(B, T, H, P, R))
            run = lambda: chunked_ssd(*args, return_final_state=True)  # noqa: E731
        elif case == "chunked_bwd":
            from . import _lib

            B, T, H, P, N, R = 2, 4096, 24, 64, 128, 2
            r = lambda *sh: torch.randn(*sh, device="cuda", generator=g).to(torch.bfloat16)  # noqa: E731
            f = lambda *sh: torch.randn(*sh, device="cuda", generator=g)  # noqa: E731
            args = (r(B, T, H, P, R), r(B, T, H, P, R), r(B, T, H, N, R), r(B, T, H, N, R), r(B, T, H, N, R),
                    torch.rand(B, T, H, device="cuda", generator=g) * 0.1, -torch.rand(H, device="cuda", generator=g),
                    torch.randn(H, device="cuda", generator=g), r(B, T, H, P, R), r(B, T, H, P, R), f(B, H, P, N),
                    f(B, H, P, N))
            run = lambda: _lib.chunked_ssd_bwd(*args)  # noqa: E731
        elif case == "in_proj":
            m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
            x = torch.randn(16, 4096, 768, device="cuda", generator=g).to(torch.bfloat16)
            run = lambda: m._project(x)  # noqa: E731
        elif case == "decode":
            from .block import KulaMambaLM
            from .decode import GraphDecoder

            lm = KulaMambaLM(vocab_size=32000, d_model=768, n_layers=24, d_state=128, headdim=64, mimo_rank=2,
                             residual_scale="depth").cuda().to(torch.bfloat16).eval()
            ids = torch.randint(0, 32000, (256, 16), device="cuda", generator=g)
            dec = GraphDecoder(lm, batch_size=256, max_new_tokens=2 + reps)
            dec.prefill(ids)
            dec.decode(1)  # captures the step graph
            torch.cuda.synchronize()
            for _ in range(reps):
                dec.decode(1)
            torch.cuda.synchronize()
            return
        elif case == "step":
            m = KulaMamba(d_model=768, d_state=128, headdim=64, mimo_rank=2).cuda().to(torch.bfloat16).eval()
            B = 256
            st = m.allocate_inference_state(B, compact=True)
            proj = m.in_proj(torch.randn(B, 768, device="cuda", generator=g).to(torch.bfloat16))
            y = torch.empty(B, m.nheads * m.headdim, device="cuda", dtype=torch.bfloat16)
            d = m._dims()
            dims = (d["H"], d["P"], d["N"], d["R"], d["G"], d["trapezoidal"], d["complex_ssm"], d["norm_eps"])
            ws = [None]

            def run():
                ws[0] = ops.step_ssm_compact_(m._param_tensors(), dims, proj, st["h"], st["prev_B"], st["prev_x"],
                                              st["angle"], y, workspace=ws[0])
        else:
            raise ValueError(case)
        for _ in range(1 + reps):
            run()
        torch.cuda.synchronize()


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="profiling helpers")
    ap.add_argument("what", choices=["train", "cfg3", "chunked", "chunked_bwd", "step", "fp32", "in_proj", "decode"])
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seqlen", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    if args.what == "train":
        print(train_step_profile(args.batch, args.seqlen))
    else:
        kernel_workload(args.what, args.reps)
