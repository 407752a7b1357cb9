"""RNGD KV connector on B200: a real vLLM KVConnectorBase_V1 subclass
(API of src/rngd_pd/connector/rngd_kv.py:27-169).

Dual construction exactly as the reference:
  * vLLM:        RngdKVConnector(vllm_config, role, kv_cache_config)
  * standalone:  RngdKVConnector(KVConnectorRole.WORKER, req_id="r1", transport=tr, n_layers=32)

The transport is injected, or named ($AIRM_KV_TRANSPORT / kv_transport=) through
select_transport, or in-process.  Host arrays travel as the reference's wire bytes
(push/pull, bf16 or fp16); torch tensors on a byte transport (shm, tcp) are staged as the
same bytes from their own 16-bit values, and registered torch buffers are filled from them
the same way (a bf16 tensor on the bf16 wire moves as raw bits both ways).  Device tensors handed to save_kv_layer go through a
transport's device path when it has one (`nvlink`: peer-to-peer stores straight into
the decode side's leased cache lane), and wait_for_layer_load then waits for that
layer's completion flag instead of pulling bytes.
"""
import os
from dataclasses import dataclass, field

import numpy as np

from rngd_pd.connector.transport import (InProcTransport, Transport, deser, deser_into, select_transport, ser,
                                         ser_tensor)

from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                               KVConnectorRole)


@dataclass
class RngdKVConnectorMetadata(KVConnectorMetadata):
    """Scheduler -> worker KV-transfer instructions for one step (rngd_kv.py:27-34)."""
    req_id: str = ""
    load_layers: list = field(default_factory=list)
    save_layers: list = field(default_factory=list)
    num_external_tokens: int = 0
    remote: str = ""


def _is_device(x):
    return hasattr(x, "is_cuda") and x.is_cuda


class RngdKVConnector(KVConnectorBase_V1):
    """vLLM KVConnectorBase_V1 subclass for PD disaggregation on B200."""

    def __init__(self, *args, req_id="r0", transport: Transport = None, n_layers=0, kv_transport=None, **kw):
        if args and isinstance(args[0], KVConnectorRole):
            role = args[0]
            if len(args) > 1 and isinstance(args[1], str):
                req_id = args[1]
            if len(args) > 2 and args[2] is not None:
                transport = args[2]
            if len(args) > 3:
                n_layers = args[3]
            self._connector_metadata = None
            self._vllm_config = None
            self._kv_transfer_config = None
            self._kv_cache_config = None
            self._role = role
        else:
            vllm_config = args[0]
            role = args[1] if len(args) > 1 else kw.get("role")
            kv_cache_config = args[2] if len(args) > 2 else kw.get("kv_cache_config")
            super().__init__(vllm_config, role, kv_cache_config)
            xfer = getattr(self._kv_transfer_config, "kv_connector_extra_config", {}) or {}
            req_id = xfer.get("req_id", req_id)
            n_layers = xfer.get("n_layers", n_layers)
            kv_transport = xfer.get("kv_transport", kv_transport)
        self.req_id = req_id
        self.n_layers = n_layers
        if transport is None and (kv_transport or os.environ.get("AIRM_KV_TRANSPORT")):
            transport = select_transport(kv_transport)
        self.t = transport or InProcTransport()
        self._kv_caches = None
        self._saved = {}
        self._loading = []

    @property
    def role(self):
        return self._role

    # ---------------------------------------------------------- scheduler side
    def get_num_new_matched_tokens(self, request, num_computed_tokens):
        n = getattr(request, "kv_ready_tokens", 0)
        extra = max(0, n - num_computed_tokens)
        return (extra if extra > 0 else None, extra > 0)

    def update_state_after_alloc(self, request, blocks, num_external_tokens):
        self._pending_alloc = (getattr(request, "request_id", self.req_id), num_external_tokens)

    def build_connector_meta(self, scheduler_output):
        layers = [f"layer.{i}" for i in range(self.n_layers)]
        is_worker = self._role == KVConnectorRole.WORKER
        return RngdKVConnectorMetadata(req_id=self.req_id, save_layers=layers if is_worker else [],
                                       load_layers=layers, num_external_tokens=self.n_layers)

    # ------------------------------------------------------------- worker side
    def register_kv_caches(self, kv_caches):
        """Bind the local KV buffers: vLLM's dict[layer_name -> tensor], or (K_list, V_list) by layer,
        or (K, V) device caches [L][Bcap][NKV][S][HD] a device transport writes into."""
        self._kv_caches = kv_caches
        if isinstance(kv_caches, dict) and self.n_layers == 0:
            self.n_layers = len(kv_caches)
        if (isinstance(kv_caches, (tuple, list)) and len(kv_caches) == 2 and all(_is_device(c) for c in kv_caches)
                and kv_caches[0].dim() == 5 and hasattr(self.t, "bind_cache")):
            self.t.bind_cache(kv_caches[0], kv_caches[1])

    @staticmethod
    def _split(kv_layer):
        if isinstance(kv_layer, (tuple, list)) and len(kv_layer) == 2:
            return kv_layer[0], kv_layer[1]
        if kv_layer.shape[0] != 2:
            raise ValueError(f"expected stacked [2,...] kv_layer, got {tuple(kv_layer.shape)}")
        return kv_layer[0], kv_layer[1]

    @staticmethod
    def _host(x):
        """A torch tensor (any device, any float dtype) or array -> float32 numpy."""
        if hasattr(x, "detach"):
            return x.detach().float().cpu().numpy()
        return np.asarray(x)

    def save_kv_layer(self, layer_name, kv_layer, attn_metadata=None, **kwargs):
        """Push one layer's KV: device tensors through the transport's device path when it has one,
        otherwise the reference's wire bytes under `req/layer.i/{k,v}` (rngd_kv.py:122-127)."""
        k, v = self._split(kv_layer)
        if _is_device(k) and hasattr(self.t, "push_layer"):
            li = int(layer_name.split(".")[-1])
            self.t.push_layer(self.req_id, li, k.contiguous(), v.contiguous())
        elif hasattr(k, "detach"):
            self.t.push(f"{self.req_id}/{layer_name}/k", ser_tensor(k))
            self.t.push(f"{self.req_id}/{layer_name}/v", ser_tensor(v))
        else:
            self.t.push(f"{self.req_id}/{layer_name}/k", ser(self._host(k)))
            self.t.push(f"{self.req_id}/{layer_name}/v", ser(self._host(v)))
        self._saved[layer_name] = True

    def wait_for_save(self):
        """Pushes are stream-ordered (device) or synchronous (host): nothing to wait for."""
        return

    def start_load_kv(self, forward_context=None, **kwargs):
        meta = self._connector_metadata
        self._loading = list(getattr(meta, "load_layers", [])) if meta else \
            [f"layer.{i}" for i in range(self.n_layers)]

    def wait_for_layer_load(self, layer_name):
        """Block until this layer's KV is present (rngd_kv.py:139-166).  Device transports:
        wait on the layer's completion flag (the bytes are already in the bound cache lane) and
        return the lane's (k, v) views.  Host transports: pull, decode and write into the
        registered buffers (torch buffers are filled in place by deser_into and returned).
        Timeout: $PD_KV_PULL_TIMEOUT (default 5 s) -> TimeoutError."""
        t = float(os.environ.get("PD_KV_PULL_TIMEOUT", "5"))
        li = int(layer_name.split(".")[-1])
        if hasattr(self.t, "lane_views") and getattr(self.t, "_cache", None) is not None:
            self.t.wait(self.req_id, layer0=li, layer1=li + 1, timeout=t)
            K, V = self.t.lane_views(self.req_id)
            return K[li], V[li]
        kb = self.t.pull(f"{self.req_id}/{layer_name}/k", timeout=t)
        vb = self.t.pull(f"{self.req_id}/{layer_name}/v", timeout=t)
        dst = None
        if isinstance(self._kv_caches, dict):
            dst = self._kv_caches.get(layer_name)
        elif self._kv_caches is not None:
            dst = (self._kv_caches[0][li], self._kv_caches[1][li])
        if dst is not None and hasattr(dst[0], "detach"):
            return deser_into(kb, dst[0]), deser_into(vb, dst[1])
        k, v = deser(kb), deser(vb)
        if dst is not None:
            dst[0][:] = k
            dst[1][:] = v
        return k, v

    def get_finished(self, finished_req_ids):
        return (None, None)
