"""SM clocks, power and throttle reasons sampled during a timed region (read-only: nothing is changed on the GPU).

NVML queries (nvidia-ml-py) every 10 ms on a thread, plus one synchronous sample when the region starts and one
when it stops, so that even a region shorter than one interval carries clocks; nvidia-smi at 200 ms where NVML is
not importable."""
import statistics
import subprocess
import threading
import time

NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def _nvml_handle(dev):
    """NVML handle of CUDA device `dev` (matched by UUID, so CUDA_VISIBLE_DEVICES orderings do not matter)."""
    import pynvml
    pynvml.nvmlInit()
    try:
        import torch
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    except Exception:
        return pynvml.nvmlDeviceGetHandleByIndex(dev)


class Clocks:
    """Samples of SM clock, power and throttle reasons during the timed region of CUDA device `dev`."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    PERIOD = 0.010

    def __init__(self, dev):
        self.dev, self.samples, self.proc, self.h, self.th = dev, [], None, None, None
        self._stop = threading.Event()
        try:
            self.h = _nvml_handle(dev)
        except Exception:
            self.h = None

    def _nvml_sample(self):
        import pynvml
        h = self.h
        reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
        bits = [pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap]
        self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                             float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)),
                             pynvml.nvmlDeviceGetPowerUsage(h) / 1e3,
                             {n for n, b in zip(NAMES, bits) if reasons & b}))

    def _nvml_loop(self):
        while not self._stop.wait(self.PERIOD):
            try:
                self._nvml_sample()
            except Exception:
                return

    def _smi_loop(self):
        for line in self.proc.stdout:
            r = [c.strip() for c in line.split(",")]
            if len(r) > 8 and r[1].replace(".", "").isdigit() and r[2].replace(".", "").isdigit():
                self.samples.append((float(r[1]), float(r[2]), None,
                                     {n for n, v in zip(NAMES, r[5:9]) if v.lower() == "active"}))

    def start(self):
        if self.h is not None:
            try:
                self._nvml_sample()
                self.th = threading.Thread(target=self._nvml_loop, daemon=True)
                self.th.start()
                return
            except Exception:
                self.h = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._smi_loop, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None

    def stop(self):
        t0 = time.perf_counter()
        if self.h is not None:
            try:
                self._nvml_sample()
            except Exception:
                pass
            self._stop.set()
            if self.th:
                self.th.join(1.0)
        elif self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm = [s[0] for s in self.samples]
        mx = [s[1] for s in self.samples]
        pw = [s[2] for s in self.samples if s[2] is not None]
        reasons = set().union(*[s[3] for s in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_median": statistics.median(pw) if pw else None,
                "source": "nvml 10 ms" if self.h is not None else "nvidia-smi 200 ms",
                "stop_overhead_s": round(time.perf_counter() - t0, 4)}
