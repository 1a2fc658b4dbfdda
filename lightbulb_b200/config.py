"""Typed configuration for models, the KV cache, the scheduler and the server.

Model presets mirror the Llama-family configs the reference ships
(``src/model/custom_transformer.rs:21-65`` ``llama_7b``/``llama2_7b``/``llama3_8b``) plus the
shapes named by the benchmark configs (TinyLlama, Phi-3-mini, Llama-3-70B, Llama-3.2-1B).
Server defaults follow ``src/main.rs:24-52`` (batch 16, ctx 4096) and the chunked-prefill
defaults follow ``src/model/chunked_prefill.rs:39-57`` (chunk 512).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class ModelConfig:
    """Architecture of a Llama-family decoder (RMSNorm, RoPE, GQA, SwiGLU)."""

    name: str = "llama"
    vocab_size: int = 32000
    hidden_size: int = 2048
    intermediate_size: int = 5632
    num_layers: int = 22
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 0  # 0 -> hidden_size // num_heads
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    bos_token_id: int = 1
    eos_token_id: int | list[int] = 2
    # Qwen3: per-head RMSNorm of q and k (weights of width head_dim) before RoPE
    # (reference src/model/awq_qwen3.rs:188-189,259-267)
    qk_norm: bool = False

    def __post_init__(self) -> None:
        if self.head_dim == 0:
            self.head_dim = self.hidden_size // self.num_heads
        assert self.num_heads % self.num_kv_heads == 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def head_dim_padded(self) -> int:
        """Head width of the device layout.  The attention kernels are built for 128-wide heads;
        narrower heads (TinyLlama / Llama-3.2-1B 64, Phi-3 96) are zero-padded to 128: the
        padded q / k / v lanes stay exactly zero, so scores and outputs are unchanged."""
        if self.head_dim > 128 or self.head_dim % 16:
            raise ValueError(f"head_dim {self.head_dim}: supported are multiples of 16 up to 128")
        return 128

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def group_size(self) -> int:
        return self.num_heads // self.num_kv_heads

    def num_params(self) -> int:
        h, f, v = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = h * (self.q_size + 2 * self.kv_size) + self.q_size * h + 3 * h * f + 2 * h
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * per_layer + emb + h

    def eos_ids(self) -> list[int]:
        e = self.eos_token_id
        return list(e) if isinstance(e, (list, tuple)) else [int(e)]

    # ---- HF config.json interop -------------------------------------------------------
    def to_hf_dict(self) -> dict:
        return {
            "architectures": ["Qwen3ForCausalLM" if self.qk_norm else "LlamaForCausalLM"],
            "model_type": "qwen3" if self.qk_norm else "llama",
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_norm_eps,
            "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
            "torch_dtype": "bfloat16",
            "lb200_name": self.name,
        }

    @classmethod
    def from_hf_dict(cls, d: dict) -> "ModelConfig":
        nh = int(d["num_attention_heads"])
        hs = int(d["hidden_size"])
        arch = " ".join(d.get("architectures") or []) + " " + str(d.get("model_type", ""))
        return cls(
            qk_norm="qwen3" in arch.lower(),
            name=d.get("lb200_name", d.get("model_type", "llama")),
            vocab_size=int(d["vocab_size"]),
            hidden_size=hs,
            intermediate_size=int(d["intermediate_size"]),
            num_layers=int(d["num_hidden_layers"]),
            num_heads=nh,
            num_kv_heads=int(d.get("num_key_value_heads", nh)),
            head_dim=int(d.get("head_dim", hs // nh) or hs // nh),
            rope_theta=float(d.get("rope_theta", 10000.0)),
            rms_norm_eps=float(d.get("rms_norm_eps", 1e-5)),
            max_position_embeddings=int(d.get("max_position_embeddings", 4096)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            bos_token_id=d.get("bos_token_id", 1) if d.get("bos_token_id") is not None else 1,
            eos_token_id=d.get("eos_token_id", 2) if d.get("eos_token_id") is not None else 2,
        )

    @classmethod
    def from_json(cls, path: str) -> "ModelConfig":
        with open(path) as f:
            return cls.from_hf_dict(json.load(f))


def _preset(**kw) -> ModelConfig:
    return ModelConfig(**kw)


PRESETS: dict[str, ModelConfig] = {
    # TinyLlama-1.1B shape.
    "tinyllama": _preset(name="tinyllama", vocab_size=32000, hidden_size=2048,
                         intermediate_size=5632, num_layers=22, num_heads=32, num_kv_heads=4,
                         rope_theta=1e4, rms_norm_eps=1e-5, max_position_embeddings=2048),
    # BASELINE config 2 / 5: Llama-3-8B shape.
    "llama3-8b": _preset(name="llama3-8b", vocab_size=128256, hidden_size=4096,
                         intermediate_size=14336, num_layers=32, num_heads=32, num_kv_heads=8,
                         rope_theta=5e5, rms_norm_eps=1e-5, max_position_embeddings=131072,
                         bos_token_id=128000, eos_token_id=[128001, 128009]),
    # Phi-3-mini shape (MHA).
    "phi3-mini": _preset(name="phi3-mini", vocab_size=32064, hidden_size=3072,
                         intermediate_size=8192, num_layers=32, num_heads=32, num_kv_heads=32,
                         rope_theta=1e4, rms_norm_eps=1e-5, max_position_embeddings=131072,
                         eos_token_id=[32000, 32007]),
    # speculative target / draft.
    "llama3-70b": _preset(name="llama3-70b", vocab_size=128256, hidden_size=8192,
                          intermediate_size=28672, num_layers=80, num_heads=64, num_kv_heads=8,
                          rope_theta=5e5, rms_norm_eps=1e-5, max_position_embeddings=131072,
                          bos_token_id=128000, eos_token_id=[128001, 128009]),
    "llama3.2-1b": _preset(name="llama3.2-1b", vocab_size=128256, hidden_size=2048,
                           intermediate_size=8192, num_layers=16, num_heads=32, num_kv_heads=8,
                           rope_theta=5e5, rms_norm_eps=1e-5, max_position_embeddings=131072,
                           tie_word_embeddings=True, bos_token_id=128000,
                           eos_token_id=[128001, 128009]),
    # Reference presets (custom_transformer.rs:21-65).
    "llama-7b": _preset(name="llama-7b", vocab_size=32000, hidden_size=4096,
                        intermediate_size=11008, num_layers=32, num_heads=32, num_kv_heads=32),
    "llama2-7b": _preset(name="llama2-7b", vocab_size=32000, hidden_size=4096,
                         intermediate_size=11008, num_layers=32, num_heads=32, num_kv_heads=32),
    # Qwen3-8B shape (per-head q/k RMSNorm); the reference's AwqQwen3 architecture.
    "qwen3-8b": _preset(name="qwen3-8b", vocab_size=151936, hidden_size=4096,
                        intermediate_size=12288, num_layers=36, num_heads=32, num_kv_heads=8,
                        head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6,
                        max_position_embeddings=40960, bos_token_id=151643,
                        eos_token_id=[151645, 151643], qk_norm=True),
    # Small shapes for tests.
    "qwen3-tiny-test": _preset(name="qwen3-tiny-test", vocab_size=512, hidden_size=512,
                               intermediate_size=1024, num_layers=2, num_heads=4,
                               num_kv_heads=2, head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6,
                               max_position_embeddings=4096, qk_norm=True),
    "tiny-test": _preset(name="tiny-test", vocab_size=512, hidden_size=256,
                         intermediate_size=512, num_layers=2, num_heads=8, num_kv_heads=2,
                         rope_theta=1e4, max_position_embeddings=4096),
}


def get_preset(name: str, **overrides) -> ModelConfig:
    cfg = dataclasses.replace(PRESETS[name])
    for k, v in overrides.items():
        setattr(cfg, k, v)
    cfg.__post_init__()
    return cfg


@dataclass
class CacheConfig:
    """Paged KV cache geometry. Block 16 matches the benchmark config."""

    block_size: int = 16
    num_blocks: int = 0  # 0 -> derive from free memory
    gpu_memory_utilization: float = 0.90
    enable_prefix_caching: bool = True
    kv_dtype: str = "bf16"
    # KV compression (H2O heavy hitters / StreamingLLM sinks); 0 disables.
    h2o_budget: int = 0
    h2o_recent: int = 4
    sink_tokens: int = 4
    streaming_window: int = 0
    h2o_decay: float = 0.95


@dataclass
class SchedulerConfig:
    """Continuous batching limits (token budget per step, chunked prefill)."""

    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    chunk_size: int = 512
    enable_chunked_prefill: bool = True
    max_model_len: int = 4096
    decode_priority: bool = True


@dataclass
class ParallelConfig:
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    # Row-parallel partial sums under tensor parallelism:
    #   "p2p"       row-parallel exchange over NVLink peer memory: the GEMM epilogue pushes rows
    #               to their owners, one kernel reduces + adds the residual + RMSNorm + gathers
    #               (parallel/rowpar.py);
    #   "allreduce" one-launch push all-reduce, then a separate add + RMSNorm (allreduce.py);
    #   "fused"     flag-signalled GEMM scatter + reduce/RMSNorm/all-gather (parallel/fused.py);
    #   "nccl"      NCCL all_reduce only.
    comm: str = "p2p"


@dataclass
class SpeculativeConfig:
    draft_model: Optional[str] = None
    num_speculative_tokens: int = 4
    min_acceptance: float = 0.3
    fallback_after_rounds: int = 10


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    speculative: SpeculativeConfig = field(default_factory=SpeculativeConfig)
    dtype: str = "bf16"
    device: str = "cuda"
    seed: int = 0
    use_cuda_graphs: bool = True
    # launch decode step N+1 before reading back step N's ids (host work overlaps the GPU)
    overlap_decode: bool = True
    model_path: Optional[str] = None


@dataclass
class ServerConfig:
    """Server settings; env names follow ``src/main.rs:24-52``."""

    bind_address: str = "127.0.0.1:8080"
    models_dir: str = "models"
    default_model: str = "default"
    database_url: Optional[str] = None
    jwt_secret: Optional[str] = None
    max_batch_size: int = 16
    max_context: int = 4096
    tls_cert: Optional[str] = None
    tls_key: Optional[str] = None
    tls_self_signed: bool = False
    tls_acme: Optional[object] = None      # server.tls.AcmeConfig

    @classmethod
    def from_env(cls) -> "ServerConfig":
        c = cls()
        c.bind_address = os.environ.get("LIGHTBULB_BIND_ADDRESS", c.bind_address)
        c.models_dir = os.environ.get("LIGHTBULB_MODELS_DIR", c.models_dir)
        c.default_model = os.environ.get("LIGHTBULB_DEFAULT_MODEL", c.default_model)
        c.database_url = os.environ.get("DATABASE_URL")
        c.jwt_secret = os.environ.get("LIGHTBULB_JWT_SECRET")
        c.tls_cert = os.environ.get("LIGHTBULB_TLS_CERT")
        c.tls_key = os.environ.get("LIGHTBULB_TLS_KEY")
        c.tls_self_signed = os.environ.get("LIGHTBULB_TLS_SELF_SIGNED", "0") == "1"
        from .server.tls import AcmeConfig
        c.tls_acme = AcmeConfig.from_env()
        return c
