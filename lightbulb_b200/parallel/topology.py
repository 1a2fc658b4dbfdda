"""Device and interconnect topology discovery.

Reference: ``src/multi_gpu/topology.rs:6-158`` probes ``cuda_if_available(i)``, hard-codes 80 GB
per GPU, assumes every P2P pair works and guesses NVLink (600 GB/s) only for exactly two GPUs,
then ``recommend_strategy`` picks data / tensor / pipeline parallelism.  Here every field is
measured from the system:

* GPUs, names, total / free memory from CUDA (``torch.cuda``), SM counts and compute capability;
* P2P capability per pair from ``cudaDeviceCanAccessPeer`` (``torch.cuda.can_device_access_peer``);
* NVLink per pair from NVML (``nvmlDeviceGetNvLinkState`` / ``nvmlDeviceGetNvLinkRemotePciInfo``),
  which on an NVSwitch box (B200 HGX) reports every GPU linked to the switch; the per-direction
  bandwidth is links x 50 GB/s (NVLink 5: 18 links = 900 GB/s);
* NVML is only read (no setting is changed); both probes are injectable so the logic is tested
  on CPU with fakes.

``recommend_strategy`` keeps the reference's decision structure (fits on one GPU -> replicate;
fits with TP inside the NVLink domain -> TP; else TP x PP) with real memory and link figures.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

NVLINK5_GBS_PER_LINK = 50.0   # per direction
PCIE5_X16_GBS = 64.0          # per direction


@dataclass
class GpuInfo:
    index: int
    name: str
    total_bytes: int
    free_bytes: int
    sm_count: int
    capability: tuple
    pci_bus_id: str = ""
    nvlinks: int = 0          # active NVLink links


@dataclass
class Topology:
    gpus: List[GpuInfo]
    p2p: List[List[bool]]                 # cudaDeviceCanAccessPeer
    link_gbs: List[List[float]]           # per-direction GB/s between i and j (0 on diagonal)
    nvswitch: bool = False
    notes: List[str] = field(default_factory=list)

    @property
    def num_gpus(self) -> int:
        return len(self.gpus)

    def min_free_bytes(self) -> int:
        return min((g.free_bytes for g in self.gpus), default=0)

    def nvlink_domain(self) -> List[int]:
        """GPUs connected to GPU 0 by NVLink (all of them on an NVSwitch box)."""
        if not self.gpus:
            return []
        return [0] + [j for j in range(1, self.num_gpus)
                      if self.link_gbs[0][j] > PCIE5_X16_GBS + 1]

    def to_dict(self) -> dict:
        return {"gpus": [g.__dict__ for g in self.gpus], "p2p": self.p2p,
                "link_gbs": self.link_gbs, "nvswitch": self.nvswitch, "notes": self.notes}


# ---------------------------------------------------------------------------------------
# probes (replaceable)
# ---------------------------------------------------------------------------------------
def cuda_probe() -> Dict[str, object]:
    """GPU list and P2P matrix from the CUDA runtime (through torch)."""
    import torch
    out = {"gpus": [], "p2p": []}
    if not torch.cuda.is_available():
        return out
    n = torch.cuda.device_count()
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        try:
            free, total = torch.cuda.mem_get_info(i)
        except Exception:
            free, total = p.total_memory, p.total_memory
        out["gpus"].append(GpuInfo(i, p.name, int(total), int(free), p.multi_processor_count,
                                   (p.major, p.minor)))
    out["p2p"] = [[i == j or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)]
                  for i in range(n)]
    return out


def nvml_probe(nvml=None) -> Dict[str, object]:
    """Active NVLink counts and the peer of each link (bus ids) from NVML, read only.
    ``nvml`` is the ``pynvml`` module or a fake with the same functions."""
    if nvml is None:
        try:
            import pynvml as nvml  # nvidia_ml_py
        except Exception:
            return {}
    try:
        nvml.nvmlInit()
    except Exception:
        return {}
    res = {"bus": [], "links": [], "remote": [], "nvswitch": False}
    try:
        n = nvml.nvmlDeviceGetCount()
        for i in range(n):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            bus = nvml.nvmlDeviceGetPciInfo(h).busId
            bus = bus.decode() if isinstance(bus, bytes) else bus
            res["bus"].append(bus)
            links, remotes = 0, []
            for l in range(18):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, l) != 1:
                        continue
                except Exception:
                    break
                links += 1
                try:
                    rb = nvml.nvmlDeviceGetNvLinkRemotePciInfo(h, l).busId
                    remotes.append(rb.decode() if isinstance(rb, bytes) else rb)
                except Exception:
                    remotes.append("")
            res["links"].append(links)
            res["remote"].append(remotes)
        # links whose far end is not a GPU of this box end at an NVSwitch
        gpu_bus = set(res["bus"])
        res["nvswitch"] = any(r and r not in gpu_bus for rs in res["remote"] for r in rs)
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    return res


def discover(cuda: Optional[Callable[[], dict]] = None,
             nvml: Optional[Callable[[], dict]] = None) -> Topology:
    c = (cuda or cuda_probe)()
    v = (nvml or nvml_probe)() or {}
    gpus: List[GpuInfo] = list(c.get("gpus", []))
    n = len(gpus)
    p2p = c.get("p2p") or [[i == j for j in range(n)] for i in range(n)]
    notes = []
    links = v.get("links") or []
    remote = v.get("remote") or []
    bus = v.get("bus") or []
    nvswitch = bool(v.get("nvswitch"))
    for i, g in enumerate(gpus):
        if i < len(links):
            g.nvlinks = int(links[i])
        if i < len(bus):
            g.pci_bus_id = bus[i]
    link = [[0.0] * n for _ in range(n)]
    for i in range(n):
        for j in range(n):
            if i == j:
                continue
            if nvswitch and gpus[i].nvlinks and gpus[j].nvlinks:
                # every GPU reaches every peer at its full NVLink bandwidth through the switch
                link[i][j] = min(gpus[i].nvlinks, gpus[j].nvlinks) * NVLINK5_GBS_PER_LINK
            elif i < len(remote) and j < len(bus) and bus[j] in remote[i]:
                link[i][j] = remote[i].count(bus[j]) * NVLINK5_GBS_PER_LINK
            elif p2p[i][j]:
                link[i][j] = PCIE5_X16_GBS
            else:
                link[i][j] = PCIE5_X16_GBS / 2  # staged through host memory
    if n and not v:
        notes.append("NVML unavailable: links estimated from P2P capability only")
    return Topology(gpus, p2p, link, nvswitch, notes)


# ---------------------------------------------------------------------------------------
# strategy
# ---------------------------------------------------------------------------------------
@dataclass
class Strategy:
    kind: str          # "single" | "replicate" | "tensor" | "tensor_pipeline"
    tp: int = 1
    pp: int = 1
    dp: int = 1
    reason: str = ""


def recommend_strategy(topo: Topology, weight_bytes: int, kv_bytes_needed: int = 0,
                       headroom: float = 0.9, num_heads: int = 0,
                       num_kv_heads: int = 0) -> Strategy:
    """Smallest TP degree (power of two, dividing the head counts) inside the NVLink domain
    whose per-GPU share of weights + KV fits; pipeline stages beyond that."""
    n = topo.num_gpus
    if n == 0:
        return Strategy("single", reason="no GPU")
    cap = int(topo.min_free_bytes() * headroom)
    need = weight_bytes + kv_bytes_needed
    if need <= cap:
        if n == 1:
            return Strategy("single", reason="fits on one GPU")
        return Strategy("replicate", dp=n, reason="fits on one GPU; one replica per GPU")
    domain = len(topo.nvlink_domain())

    def heads_ok(t):
        return (not num_heads or num_heads % t == 0) and (not num_kv_heads or
                                                          num_kv_heads % t == 0 or t % num_kv_heads == 0)
    t = 2
    while t <= domain:
        if heads_ok(t) and need / t <= cap:
            return Strategy("tensor", tp=t, dp=max(1, n // t),
                            reason=f"needs {need / 2**30:.1f} GiB; TP={t} inside the NVLink domain")
        t *= 2
    tp = 1
    while tp * 2 <= domain and heads_ok(tp * 2):
        tp *= 2
    pp = 2
    while pp * tp <= n:
        if need / (tp * pp) <= cap:
            return Strategy("tensor_pipeline", tp=tp, pp=pp,
                            reason=f"TP={tp} x PP={pp}: weights + KV split over {tp * pp} GPUs")
        pp += 1
    return Strategy("tensor_pipeline", tp=tp, pp=max(1, n // tp),
                    reason="does not fit even on every GPU; KV must be reduced")
