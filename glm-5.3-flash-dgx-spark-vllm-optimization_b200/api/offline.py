"""Offline entry point: ``LLM(...).generate(prompts, params)`` builds the model (a checkpoint directory in the EXL3
layout, or random-init weights of a named architecture), the GPU backend and the engine, and runs requests to
completion."""

from __future__ import annotations

import os
import time
from dataclasses import dataclass

import torch

from ..config import ModelConfig, config_by_name
from ..engine.backend import GPUBackend
from ..engine.llm import EngineConfig, LLMEngine, SamplingParams
from ..engine.tokenizer import ByteTokenizer
from ..models import weights as W
from ..models.runtime import RuntimeConfig


@dataclass
class LLMOptions:
    model: str = "tiny"                 # "tiny", "full", or a checkpoint directory
    seed: int = 0
    max_seqs: int = 4
    max_model_len: int = 8192
    page_size: int = 64
    kv_pages: int | None = None         # default: enough for max_seqs * max_model_len
    kv_cache_bytes: int | None = None   # KV budget in bytes per GPU (sets kv_pages; the reference's --kv-cache-memory)
    prefill_chunk: int = 2048
    speculative: bool = True
    k_set: tuple[int, ...] = (4, 5, 7)
    k_fixed: int | None = None
    force_accept: bool = False
    checkpoints: int = 4
    cuda_graphs: bool = True
    layers: int | None = None           # truncate the full architecture (smoke use)
    overrides: dict | None = None       # checkpoint name -> tensor or file replacing it at load
    override_sha256: dict | None = None  # checkpoint name -> expected sha256 of the override file
    vtrim_tau: float = 0.0              # verify trimming by drafter confidence (0: off)
    block_verify: bool = False          # sampled requests: block verification instead of standard
    mixed_prefill_chunk: int = 0        # prefill tokens per step while requests decode (0: the whole chunk)
    ep: bool = False                    # routed experts expert-parallel over the ranks (parallel/ep.py)
    sp_mla: bool = os.environ.get("GLM53_SP_MLA", "1") == "1"   # row-parallel MLA in sequence-parallel prefill


class LLM:
    def __init__(self, opts: LLMOptions | None = None, comm=None, rank: int = 0, world: int = 1, **kw):
        opts = opts or LLMOptions(**kw)
        self.opts = opts
        from ..utils import switches
        switches.enforce()                                        # malformed GLM53_* values stop the start
        if os.environ.get("GLM53_BOOT_CHECKS", "0") == "1":      # per-rank boot assertions (collective)
            from ..utils import boot_checks
            self.boot_report = boot_checks.run()
            boot_checks.enforce(self.boot_report)
        dev = torch.device("cuda", torch.cuda.current_device())
        if os.path.isdir(opts.model):
            cfg = W.load_config(opts.model)
            src = W.SafetensorsSource(opts.model)
        else:
            cfg = config_by_name(opts.model)
            if opts.layers:
                from ..config import full_config
                cfg = full_config(opts.layers) if opts.model in ("full", "glm53", "glm-5.3-flash") else cfg
            src = W.RandomSource(cfg, seed=opts.seed, device=dev)
        if opts.overrides:
            src = W.OverrideSource(src, opts.overrides, opts.override_sha256)
        self.cfg: ModelConfig = cfg
        t0 = time.time()
        self.weights = W.prepare(src, cfg, rank=rank, world=world, device=dev, ep=opts.ep, sp_mla=opts.sp_mla)
        self.load_s = time.time() - t0
        if opts.kv_cache_bytes and not opts.kv_pages:
            opts.kv_pages = max(1, int(opts.kv_cache_bytes // (cfg.kv_bytes_per_token() * opts.page_size)))
        pages = opts.kv_pages or max(64, opts.max_seqs * ((opts.max_model_len + opts.page_size - 1)
                                                           // opts.page_size + 2))
        kmax = max(opts.k_set) if opts.k_fixed is None else opts.k_fixed
        rc = RuntimeConfig(max_rows=max(opts.prefill_chunk, 16), max_seqs=opts.max_seqs,
                           kv_slots=pages * opts.page_size, block_size=opts.page_size,
                           max_blocks=(opts.max_model_len + opts.page_size - 1) // opts.page_size + 2,
                           decode_rows=max(16, opts.max_seqs * (kmax + 1)),
                           logit_rows=max(16, opts.max_seqs * (kmax + 1)))
        self.backend = GPUBackend(self.weights, rc, comm=comm, drafter=opts.speculative,
                                  cuda_graphs=opts.cuda_graphs, checkpoints=opts.checkpoints)
        ec = EngineConfig(max_seqs=opts.max_seqs, page_size=opts.page_size, num_pages=pages,
                          max_model_len=opts.max_model_len, prefill_chunk=opts.prefill_chunk,
                          speculative=opts.speculative, k_set=opts.k_set, k_fixed=opts.k_fixed,
                          force_accept=opts.force_accept, checkpoints=opts.checkpoints,
                          cuda_graphs=opts.cuda_graphs, vtrim_tau=opts.vtrim_tau,
                          block_verify=opts.block_verify, mixed_prefill_chunk=opts.mixed_prefill_chunk)
        self.engine = LLMEngine(self.backend, ec, eos=tuple(cfg.eos))
        self.tokenizer = ByteTokenizer(cfg.vocab)
        from ..utils.trace import maybe_attach
        self.tracer = maybe_attach(self.engine, comm, rank)          # GLM53_TRACE=<path>: per-step records

    def generate(self, prompts, params: SamplingParams | None = None) -> list[dict]:
        """prompts: strings (byte-tokenized) or token-id lists.  Returns per prompt the token ids and text."""
        ids = [self.tokenizer.encode(p) if isinstance(p, str) else list(p) for p in prompts]
        outs = self.engine.generate(ids, params or SamplingParams())
        return [{"token_ids": o, "text": self.tokenizer.decode(o)} for o in outs]
