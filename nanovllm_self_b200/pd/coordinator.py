"""Offline P/D coordinator: one prefill runner and one decode runner behind one store.

Reference: ``pd_self/coordinator.py:14-79``.  ``generate(texts, max_tokens, temperature,
ignore_eos)`` prefills everything on the prefill engine, hands the payloads over the KV
store, then decodes on the decode engine.  The two runners may share a device (the
reference's layout) or sit on two devices (``prefill_device`` / ``decode_device``).
"""
from __future__ import annotations

from ..config import EngineConfig
from ..engine.model_runner import ModelRunner
from ..parallel.state import TPState
from .decode_engine import DecodeEngine
from .kv_connector import KVConnector
from .kv_store import make_backend
from .prefill_engine import PrefillEngine


def _split_configs(config: EngineConfig, prefill_device=None, decode_device=None):
    pdev = prefill_device or config.device
    ddev = decode_device or config.device
    same = str(pdev) == str(ddev)
    util = config.gpu_memory_utilization
    pcfg = config.replace(device=pdev, gpu_memory_utilization=util / 2 if same else util)
    dcfg = config.replace(device=ddev)
    return pcfg, dcfg


def _tp_for(device):
    import torch
    dev = torch.device(device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    return TPState(device=dev)


class PDCoordinator:
    def __init__(self, config: EngineConfig, kv_backend: str = "dict", tokenizer=None,
                 prefill_device=None, decode_device=None):
        self.config = config
        if kv_backend == "dict" and str(config.device).startswith("cuda"):
            kv_backend = "device"
        self.kv_backend = make_backend(kv_backend)
        pcfg, dcfg = _split_configs(config, prefill_device, decode_device)
        self.prefill_runner = ModelRunner(pcfg, _tp_for(pcfg.device))
        self.decode_runner = ModelRunner(dcfg, _tp_for(dcfg.device))
        self.tokenizer = tokenizer
        self.producer = KVConnector(pcfg, "producer", "prefill-0", self.kv_backend)
        self.consumer = KVConnector(dcfg, "consumer", "decode-0", self.kv_backend)
        self.producer.register_model_runner(self.prefill_runner)
        self.consumer.register_model_runner(self.decode_runner)
        self.prefill_engine = PrefillEngine(pcfg, tokenizer, self.prefill_runner, self.producer)
        self.decode_engine = DecodeEngine(dcfg, tokenizer, self.decode_runner, self.consumer)
        self.prefill_engine.scheduler.eos = config.eos
        self.decode_engine.scheduler.eos = config.eos
        self._next_seq = 0

    def generate(self, texts, max_tokens: int = 64, temperature: float = 0.0, ignore_eos: bool = True):
        start = self._next_seq
        self._next_seq += len(texts)
        payloads = self.prefill_engine.run_prefill(texts, temperature, max_tokens, ignore_eos, start_seq_id=start)
        results = self.decode_engine.run_decode(payloads)
        return [results[p.request_id] for p in payloads]
