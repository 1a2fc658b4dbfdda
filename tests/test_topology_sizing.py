"""Topology discovery and sizing on CPU with fake CUDA / NVML probes (no GPU setting is read
or changed)."""
from lightbulb_b200.config import get_preset
from lightbulb_b200.engine import sizing
from lightbulb_b200.parallel.topology import GpuInfo, discover, nvml_probe, recommend_strategy

GB = 1 << 30


def _cuda8():
    gpus = [GpuInfo(i, "NVIDIA B200", 180 * GB, 170 * GB, 148, (10, 0)) for i in range(8)]
    return {"gpus": gpus, "p2p": [[True] * 8 for _ in range(8)]}


class FakeNVML:
    """Eight GPUs, 18 NVLinks each, every link ending at an NVSwitch."""

    class _Pci:
        def __init__(self, b):
            self.busId = b

    def nvmlInit(self):
        pass

    def nvmlShutdown(self):
        pass

    def nvmlDeviceGetCount(self):
        return 8

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetPciInfo(self, h):
        return self._Pci(f"0000:{h:02x}:00.0".encode())

    def nvmlDeviceGetNvLinkState(self, h, l):
        return 1

    def nvmlDeviceGetNvLinkRemotePciInfo(self, h, l):
        return self._Pci(b"0000:ff:00.0")  # switch


def test_discover_nvswitch_box():
    topo = discover(_cuda8, lambda: nvml_probe(FakeNVML()))
    assert topo.num_gpus == 8 and topo.nvswitch
    assert all(g.nvlinks == 18 for g in topo.gpus)
    assert topo.link_gbs[0][7] == 900.0 and topo.link_gbs[3][3] == 0.0
    assert topo.nvlink_domain() == list(range(8))


def test_discover_without_nvml_falls_back_to_p2p():
    topo = discover(_cuda8, lambda: {})
    assert not topo.nvswitch and topo.link_gbs[0][1] == 64.0
    assert topo.notes and "NVML" in topo.notes[0]


def test_recommend_strategy():
    topo = discover(_cuda8, lambda: nvml_probe(FakeNVML()))
    c8 = get_preset("llama3-8b")
    s = recommend_strategy(topo, sizing.weight_bytes(c8), 20 * GB)
    assert s.kind == "replicate" and s.dp == 8
    c70 = get_preset("llama3-70b")
    s = recommend_strategy(topo, sizing.weight_bytes(c70), 60 * GB, num_heads=64, num_kv_heads=8)
    assert s.kind == "tensor" and s.tp == 2
    s = recommend_strategy(topo, 2000 * GB, 0, num_heads=64, num_kv_heads=8)
    assert s.kind == "tensor_pipeline"


def test_memory_estimates_match_layouts():
    c = get_preset("llama3-8b")
    wb = sizing.weight_bytes(c)
    assert 14.5 * GB < wb < 15.5 * GB                      # 8.03 B params bf16 = 14.96 GiB
    assert sizing.kv_bytes_per_token(c) == 32 * 2 * 8 * 128 * 2
    q = sizing.weight_bytes(c, quant_bits=4)
    assert q < wb / 2
    # head padding: Phi-3 (96-wide heads) pays 128 lanes per head
    p = get_preset("phi3-mini")
    assert sizing.kv_bytes_per_token(p) == 32 * 2 * 32 * 128 * 2
    plan = sizing.plan_memory(c, 170 * GB, max_model_len=4096)
    assert plan.fits and plan.max_seqs_at_len > 256


def test_batch_adjuster_rule_and_cooldown():
    t = [0.0]
    adj = sizing.RuntimeBatchAdjuster(64, sizing.BatchSizeConfig(min_batch_size=4,
                                                                 max_batch_size=100,
                                                                 cooldown_s=1.0),
                                      clock=lambda: t[0])
    assert adj.check(90, 100, 0) == 48            # > 80 %: x3/4
    assert adj.check(90, 100, 0) is None           # cooldown
    t[0] = 2.0
    assert adj.check(10, 100, 10) is None          # queue shorter than the batch
    assert adj.check(10, 100, 500) == 60           # < 50 % and backlog: x5/4
    t[0] = 4.0
    assert adj.check(60, 100, 500) is None         # between thresholds
    adj.record_batch_memory(1000, 10)
    adj.record_batch_memory(900, 3)
    assert adj.peak_per_request == 300


def test_profile_and_auto_detect_with_fake_topology():
    topo = discover(_cuda8, lambda: nvml_probe(FakeNVML()))
    prof = sizing.HardwareProfile.detect(topo)
    assert prof.gpu_free_min == 170 * GB and prof.nvswitch
    # 70B bf16 (131 GiB) fits on one 170 GiB GPU with 16 sequences of 4k tokens, not 32
    assert sizing.recommend_model(prof, seq_len=4096, min_batch=8) == "llama3-70b"
    assert sizing.recommend_model(prof, seq_len=4096, min_batch=32) == "llama3-8b"
    sc = sizing.SystemConfig.auto_detect(seq_len=4096, model="llama3-8b", topology=topo)
    assert sc.model == "llama3-8b" and sc.batch_size > 100 and sc.plan.fits


def test_trace_categories_and_nvtx_noop():
    from lightbulb_b200.utils import trace
    trace.configure(debug="kv,spec", nvtx=False)
    assert trace.enabled("kv") and trace.enabled("spec") and not trace.enabled("decode")
    with trace.nvtx_range("x"):
        trace.debug("kv", "message %d", 1)
    trace.configure(debug="all", nvtx=False)
    assert all(trace.enabled(c) for c in trace.CATEGORIES)
    trace.configure(debug="", nvtx=False)
