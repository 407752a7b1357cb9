"""rm-core v0.1.1 protocol types, for hosts without the `rm_core` package.

The reference pins `rm-core @ git+https://github.com/ai-computing/rm-core@v0.1.1`
(pyproject.toml:9-12) and imports these names from it (src/rngd_pd/airm.py:43-46,
src/rngd_pd/connector/transport.py:252,271).  That package is not vendored and is
not installed here, so this module restates the subset of its protocol the KV
transports use, with the semantics their call sites rely on.  When `rm_core` is
importable, rngd_pd uses it instead (see rngd_pd.airm).
"""
from dataclasses import dataclass, field


class ContractError(ValueError):
    """A caller broke the transport contract (wrong sizes, bad arguments)."""


class TransportError(RuntimeError):
    """A transfer could not be planned or did not complete."""


DTYPE_BYTES = {"bf16": 2, "fp16": 2, "fp8": 1, "int8": 1, "fp32": 4}
TIER_KINDS = ("host-dram", "device-hbm", "remote")


@dataclass(frozen=True)
class KVLayout:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    dtype: str = "bf16"

    def validate(self):
        if min(self.num_layers, self.num_kv_heads, self.head_dim) <= 0:
            raise ContractError(f"non-positive KV layout {self}")
        if self.dtype not in DTYPE_BYTES:
            raise ContractError(f"unknown KV dtype {self.dtype!r}")
        return self

    def bytes_per_token(self):
        """K and V for every layer and head of one token."""
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * DTYPE_BYTES[self.dtype]


@dataclass(frozen=True)
class MemoryTier:
    name: str
    kind: str
    capacity_bytes: int
    location: str = ""

    def validate(self):
        if self.kind not in TIER_KINDS:
            raise ContractError(f"unknown tier kind {self.kind!r}")
        if self.capacity_bytes <= 0:
            raise ContractError(f"tier {self.name} has no capacity")
        return self


@dataclass
class TransferPlan:
    request_id: str
    src: MemoryTier
    dst: MemoryTier
    src_layout: KVLayout
    dst_layout: KVLayout
    tokens: tuple
    nbytes: int
    detail: dict = field(default_factory=dict)


@dataclass(frozen=True)
class TransferHandle:
    request_id: str
    transport: str
    token: str


@dataclass
class TransferResult:
    request_id: str
    ok: bool
    nbytes: int
    seconds: float
    error: str = None


# name -> (unit, direction, help), the subset of rm-core's METRICS this package emits: the
# transports' per-transfer figures and the serving summary (rngd_pd.airm.summarize)
METRICS = {"kv_transfer_ms": ("ms", "lower", "KV handoff time per transfer"),
           "kv_transfer_gbps": ("GB/s", "higher", "KV handoff payload bandwidth"),
           "ttft_p90_ms": ("ms", "lower", "time to first token, 90th percentile"),
           "tpot_p90_ms": ("ms", "lower", "time per output token after the first, 90th percentile"),
           "tok_s": ("tok/s", "higher", "generated tokens per second over the window")}


@dataclass
class Measurement:
    name: str
    value: float
    tags: dict = field(default_factory=dict)

    @property
    def unit(self):
        return METRICS[self.name][0]

    def validate(self):
        if self.name not in METRICS:
            raise ContractError(f"unknown measurement {self.name!r}")
        if not isinstance(self.value, (int, float)) or self.value != self.value:
            raise ContractError(f"measurement {self.name} has no numeric value")
        return self


def prometheus_name(name):
    return "airm_" + name
