"""Host preflight: per-GPU health bench, cross-GPU outliers, host facts, thresholds -> a verdict and header facts.

Reference: `modules/metrics/preflight.py:142-253` (orchestration, thresholds), `gpu.py:142-317` (bf16 matmul
TFLOPS, decode-shaped weight-stream GB/s, power limit, temperature and throttle reasons per GPU,
cross-GPU outlier detection) and `network.py:20-87` (download speed).

Per GPU: bf16 GEMM throughput (8192^3 by default, CUDA events around a timed loop after warm-up),
HBM copy bandwidth (a device-to-device copy of a buffer larger than L2), and a decode-shaped weight stream
(M = 48 rows times a set of weight matrices that together exceed L2, the memory-bound GEMM shape of
speculative verification). NVML is read only: name, power limit, temperature, SM clock and the active
clock-event reasons. Outliers: a GPU below `outlier_frac` of the median of its peers is flagged.
Nothing here changes any GPU setting.

    python -m phung5_b200.utils.preflight --out preflight.json [--quick]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from dataclasses import asdict, dataclass, field
from typing import Callable, Dict, List, Optional

# family thresholds: (min bf16 TFLOPS, min copy GB/s), a healthy part measures well above both
FAMILY_MIN = {"B200": (1000.0, 5000.0), "H200": (530.0, 3000.0), "H100": (250.0, 1100.0)}
THROTTLE_BAD = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "hw_power_brake_slowdown")


@dataclass
class GPUResult:
    index: int
    name: str = "?"
    tflops: Optional[float] = None
    copy_gbs: Optional[float] = None
    stream48_gbs: Optional[float] = None
    power_limit_w: Optional[float] = None
    power_w: Optional[float] = None
    temp_c: Optional[int] = None
    sm_mhz: Optional[int] = None
    sm_max_mhz: Optional[int] = None
    reasons: List[str] = field(default_factory=list)
    error: Optional[str] = None
    flags: List[str] = field(default_factory=list)


# ------------------------------------------------------------------------------------------------------ NVML


class NvmlReader:
    """Read-only NVML queries (pynvml from nvidia_ml_py). `lib` can be a fake with the same functions."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, lib=None):
        if lib is None:
            import pynvml as lib  # noqa: N813
        self.nv = lib
        self.nv.nvmlInit()

    def count(self) -> int:
        return int(self.nv.nvmlDeviceGetCount())

    def read(self, i: int) -> dict:
        nv = self.nv
        h = nv.nvmlDeviceGetHandleByIndex(i)
        name = nv.nvmlDeviceGetName(h)
        name = name.decode() if isinstance(name, bytes) else str(name)
        out = {"name": name}
        for key, fn in (("power_limit_w", lambda: nv.nvmlDeviceGetEnforcedPowerLimit(h) / 1000.0),
                        ("power_w", lambda: nv.nvmlDeviceGetPowerUsage(h) / 1000.0),
                        ("temp_c", lambda: int(nv.nvmlDeviceGetTemperature(h, 0))),
                        ("sm_mhz", lambda: int(nv.nvmlDeviceGetClockInfo(h, 1))),
                        ("sm_max_mhz", lambda: int(nv.nvmlDeviceGetMaxClockInfo(h, 1)))):
            try:
                out[key] = fn()
            except Exception:  # noqa: BLE001 - a missing counter is reported as unknown
                out[key] = None
        try:
            mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
        except Exception:  # noqa: BLE001
            try:
                mask = int(nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))
            except Exception:  # noqa: BLE001
                mask = 0
        out["reasons"] = [n for b, n in self.REASONS.items() if mask & b]
        return out


# ------------------------------------------------------------------------------------------------- GPU bench


def bench_gpu(index: int, n: int = 8192, seconds: float = 2.0, copy_mib: int = 2048, stream_gb: float = 1.0) -> dict:
    import torch
    dev = torch.device(f"cuda:{index}")
    torch.cuda.set_device(dev)
    out = {}
    a = torch.randn(n, n, device=dev, dtype=torch.bfloat16)
    b = torch.randn(n, n, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        a @ b
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    iters, t0 = 0, time.monotonic()
    s.record()
    while time.monotonic() - t0 < seconds:
        for _ in range(10):
            a @ b
        iters += 10
        torch.cuda.synchronize(dev)
    e.record()
    e.synchronize()
    out["tflops"] = 2.0 * n ** 3 * iters / (s.elapsed_time(e) / 1e3) / 1e12
    del a, b
    src = torch.empty(copy_mib * 2 ** 20, dtype=torch.uint8, device=dev)
    dst = torch.empty_like(src)
    dst.copy_(src)
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(10):
        dst.copy_(src)
    e.record()
    e.synchronize()
    out["copy_gbs"] = 2 * src.numel() * 10 / (s.elapsed_time(e) / 1e3) / 1e9
    del src, dst
    k = 8192
    nw = max(2, int(stream_gb * 2 ** 30 // (k * k * 2)))
    ws = [torch.randn(k, k, device=dev, dtype=torch.bfloat16) for _ in range(nw)]
    x = torch.randn(48, k, device=dev, dtype=torch.bfloat16)
    for w in ws:
        x @ w
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(3):
        for w in ws:
            x @ w
    e.record()
    e.synchronize()
    out["stream48_gbs"] = 3 * nw * k * k * 2 / (s.elapsed_time(e) / 1e3) / 1e9
    return out


def family_min(name: str, cfg: Optional[dict] = None) -> tuple:
    cfg = cfg or {}
    d = next((v for k, v in FAMILY_MIN.items() if k in (name or "").upper()), (30.0, 0.0))
    return (cfg.get("min_tflops") or d[0], cfg.get("min_hbm_gbs") or d[1])


def flag_outliers(results: List[GPUResult], key: str, frac: float = 0.85) -> None:
    vals = [getattr(r, key) for r in results if getattr(r, key) is not None]
    if len(vals) < 2:
        return
    med = statistics.median(vals)
    for r in results:
        v = getattr(r, key)
        if v is not None and v < frac * med:
            r.flags.append(f"{key}_outlier({v:.0f}<{frac:.2f}x{med:.0f})")


def run_preflight(n_gpus: Optional[int] = None, nvml=None, bench: Optional[Callable[[int], dict]] = None,
                  thresholds: Optional[dict] = None, outlier_frac: float = 0.85) -> dict:
    thresholds = thresholds or {}
    if nvml is None:
        try:
            nvml = NvmlReader()
        except Exception:  # noqa: BLE001 - no NVML: bench only
            nvml = None
    if n_gpus is None:
        if nvml is not None:
            n_gpus = nvml.count()
        else:
            import torch
            n_gpus = torch.cuda.device_count()
    bench = bench or bench_gpu
    results: List[GPUResult] = []
    for i in range(n_gpus):
        r = GPUResult(index=i)
        if nvml is not None:
            try:
                for k, v in nvml.read(i).items():
                    setattr(r, k, v)
            except Exception as e:  # noqa: BLE001
                r.flags.append(f"nvml_error({type(e).__name__})")
        try:
            for k, v in bench(i).items():
                setattr(r, k, v)
        except Exception as e:  # noqa: BLE001
            r.error = f"{type(e).__name__}: {str(e)[:160]}"
            r.flags.append("bench_failed")
        if nvml is not None:
            try:
                r.reasons = sorted(set(r.reasons) | set(nvml.read(i).get("reasons", [])))
            except Exception:  # noqa: BLE001
                pass
        results.append(r)
    for key in ("tflops", "copy_gbs", "stream48_gbs"):
        flag_outliers(results, key, outlier_frac)
    bad = 0
    for r in results:
        mt, mb = family_min(r.name, thresholds)
        if r.tflops is not None and r.tflops < mt:
            r.flags.append(f"tflops<{mt:.0f}")
        if r.copy_gbs is not None and mb and r.copy_gbs < mb:
            r.flags.append(f"copy<{mb:.0f}")
        mp = thresholds.get("min_power_limit_w")
        if mp and r.power_limit_w is not None and r.power_limit_w < mp:
            r.flags.append(f"power_limit<{mp:.0f}")
        if any(x in THROTTLE_BAD for x in r.reasons):
            r.flags.append("throttled")
        bad += 1 if (r.flags or r.error) else 0
    cpu_quota = None
    try:
        from ..app.batch_stats import cpu_quota as _q
        cpu_quota = _q()
    except Exception:  # noqa: BLE001
        pass
    diag = {"gpus": n_gpus, "tflops": [r.tflops for r in results], "hbm_gbs": [r.copy_gbs for r in results],
            "power_w": [r.power_limit_w for r in results], "gpu_sm": [r.sm_max_mhz for r in results],
            "gpu_temp": max((r.temp_c for r in results if r.temp_c is not None), default="?"),
            "gpu_thr": sum(1 for r in results if "throttled" in r.flags), "gpu_bad": bad,
            "cpu_quota": f"{cpu_quota:.1f}" if cpu_quota else "?", "nproc": os.cpu_count()}
    return {"ok": bad == 0, "gpus": [asdict(r) for r in results], "diag": diag}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="preflight.json")
    ap.add_argument("--quick", action="store_true", help="smaller GEMM and copies (a few seconds per GPU)")
    ap.add_argument("--min-tflops", type=float)
    ap.add_argument("--min-hbm-gbs", type=float)
    ap.add_argument("--min-power-limit-w", type=float)
    args = ap.parse_args(argv)
    bench = (lambda i: bench_gpu(i, n=4096, seconds=0.5, copy_mib=512, stream_gb=0.5)) if args.quick else None
    res = run_preflight(bench=bench, thresholds={"min_tflops": args.min_tflops, "min_hbm_gbs": args.min_hbm_gbs,
                                                 "min_power_limit_w": args.min_power_limit_w})
    with open(args.out, "w") as f:
        json.dump(res, f, indent=1)
    print(json.dumps({"ok": res["ok"], "diag": res["diag"]}))


if __name__ == "__main__":
    main()
