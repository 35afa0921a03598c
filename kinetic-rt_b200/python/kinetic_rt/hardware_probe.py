"""Hardware discovery (python/kinetic_rt/hardware_probe.py of the reference):
(topology, backend, target) with target "sm{major}{minor}" on CUDA devices,
overridable through KINETIC_TARGET."""
import os


def probe_hardware():
    forced = os.environ.get("KINETIC_TARGET")
    if forced:
        backend = "CUDA" if "sm" in forced else ("ROCm" if "gfx" in forced else "CPU")
        return "1x Overridden GPU", backend, forced
    try:
        import torch
    except ImportError:
        return "CPU Only (Headless)", "CPU", "CPU"
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        name = torch.cuda.get_device_name(0)
        if getattr(torch.version, "hip", None):
            arch = getattr(torch.cuda.get_device_properties(0), "gcnArchName", None)
            if not arch:
                raise RuntimeError("Architecture could not be dynamically probed.")
            return f"{n}x {name}", "ROCm", arch.split(":")[0]
        major, minor = torch.cuda.get_device_capability(0)
        return f"{n}x {name} (Compute {major}.{minor})", "CUDA", f"sm{major}{minor}"
    return "CPU Only (Headless)", "CPU", "CPU"


def get_topology_string():
    topology, backend, target = probe_hardware()
    if backend == "CPU":
        return "[Kinetic-RT] Hardware Detected: CPU Only (Headless)"
    return f"[Kinetic-RT Init] Detected Topology: {topology} | Backend: {backend} | Target: {target}"
