"""Public facade, same names and defaults as evspark/api.py:31-216.

    from evspark_b200 import EvSpark
    es = EvSpark.load(model_name="evo2_7b")            # random-init target + drafter of that shape
    res = es.generate("ACGT..." * 16, n_tokens=1024)   # sampling, T=1.0, top_k=4
    g = es.generate(prompt, greedy=True)
    nat = es.generate_native(prompt, greedy=True)
    assert g.ids.tolist() == nat.ids.tolist()

Real Evo2 weights and trained drafter checkpoints are not available offline: the target is a
seeded random-init StripedHyena2 of the named shape, and the drafter is loaded from a local
checkpoint of the reference's .pt schema when ``ckpt`` is a file, else seeded random-init.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

DEFAULT_CKPT = "L27_g12_150M_s1"


def clean_prompt(seq: str) -> str:
    """Upper-case and validate ACGTN; reject short prompts (evspark/api.py:31-39)."""
    seq = "".join(seq.split()).upper()
    bad = sorted(set(seq) - set("ACGTN"))
    if bad:
        raise ValueError(f"prompt contains non-ACGTN characters: {bad}")
    if len(seq) < 64:
        raise ValueError("prompt too short (<64 bp); give the model some context")
    return seq


def ids_to_text(ids) -> str:
    """token id = ASCII byte (CharLevelTokenizer convention)."""
    arr = np.clip(np.asarray(ids, dtype=np.int64).ravel(), 0, 255)
    return bytes(arr.tolist()).decode("ascii", errors="replace")


def tokenize(seq: str) -> np.ndarray:
    return np.frombuffer(seq.encode("ascii"), dtype=np.uint8).astype(np.int64)


@dataclass
class GenerateResult:
    text: str
    ids: np.ndarray
    mode: str
    speculative: bool
    n_tokens: int
    wall_s: float
    tok_s: float
    mean_tau: float | None = None
    n_rounds: int | None = None
    extra: dict = field(default_factory=dict)


def _init_graph_capture(device) -> None:
    """The first CUDA-graph capture of a process initialises the runtime's graph machinery (tens of
    milliseconds); do it once at load time, not inside the first generate call (whose rounds capture
    the drafter call as a graph)."""
    import torch

    dev = torch.device(device)
    if dev.type != "cuda" or not torch.cuda.is_available():
        return
    with torch.cuda.device(dev):
        x = torch.zeros(1, device=dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            x.add_(1.0)
        g.replay()
        torch.cuda.synchronize(dev)
        del g


class EvSpark:
    """state_seqlen: positions of the decode state allocated here and reused by every generate call
    whose prompt + tokens + gamma fit (a serving engine's preallocated caches: a call then allocates
    no device memory); a longer call allocates a larger state, which is kept instead.  0: allocate
    the state on first use."""

    def __init__(self, model, nd, device: str = "cuda:0", *, state_seqlen: int = 4096):
        self.model = model
        self._nd = nd
        self.device = device
        self._state = None
        _init_graph_capture(device)
        if state_seqlen > 0:
            self._state = self._new_state(int(state_seqlen))

    def _new_state(self, max_seqlen: int):
        from evspark_b200.specdec.block.loop import PREFILL_CHUNK_MAX

        # the largest prefill chunk, so that every prompt is prefilled in the chunks a fresh state of
        # its own length would use (the results do not depend on the chunking either)
        return self.model.initialize_inference_params(max_seqlen=max_seqlen, max_batch=1,
                                                      max_chunk=PREFILL_CHUNK_MAX)

    def _decode_state(self, need: int):
        """The kept decode state, reset to length 0, or a new one when `need` positions do not fit."""
        if self._state is not None and self._state.max_seqlen >= need:
            self._state.batch = 1
            self._state.set_offset(0)
            return self._state
        if self._state is not None:
            self._state.close()
            self._state = None
        self._state = self._new_state(need)
        return self._state

    @classmethod
    def load(cls, ckpt: str | None = DEFAULT_CKPT, model_name: str = "evo2_7b", device: str = "cuda:0",
             use_kernels: bool = True, *, seed: int = 20260820, drafter_seed: int = 20260830,
             max_chunk: int = 32) -> "EvSpark":
        import torch

        from evspark_b200.config import DRAFTERS, target_config
        from evspark_b200.drafter import DeviceDrafter, load_checkpoint, layer_index
        from evspark_b200.model import TargetModel, require_device
        from evspark_b200.specdec.block.neural_draft import NeuralDraftModel

        if not use_kernels:
            raise ValueError("evspark_b200 has one compute path: the sm_100a kernels (use_kernels=True)")
        require_device(device)
        cfg = target_config(model_name)
        path = Path(str(ckpt)) if ckpt else None
        if path is not None and path.is_file():
            dcfg_layers = torch.load(path, map_location="cpu")["scheme"]
            from evspark_b200.drafter import SCHEME_LAYERS

            layers = SCHEME_LAYERS[dcfg_layers]
        else:
            layers = DRAFTERS[model_name].inject_layers
        init_on = "cuda" if cfg.d_model >= 1024 else "cpu"
        model = TargetModel.random(cfg, seed=seed, device=device, init_on=init_on,
                                   capture_layers=tuple(layer_index(n) for n in layers), max_chunk=max_chunk)
        if path is not None and path.is_file():
            drafter, layers, meta = load_checkpoint(str(path), cfg.d_model, device=device)
        else:
            dcfg = DRAFTERS[model_name]
            drafter = DeviceDrafter.random(dcfg, seed=drafter_seed, embed=model.weights["embed"], device=device,
                                           init_on=init_on)
        nd = NeuralDraftModel(model, drafter, tuple(layers))
        return cls(model, nd, device)

    @property
    def gamma(self) -> int:
        return int(self._nd.gamma)

    def _ids(self, prompt: str):
        import torch

        seq = clean_prompt(prompt)
        return seq, torch.as_tensor(tokenize(seq)[None], device=self.model.device)

    def _ids_pinned(self, prompt: str):
        """The prompt's ids on the host (pinned) and on the device: one host-to-device copy."""
        import torch

        from evspark_b200 import _native as N

        seq = clean_prompt(prompt)
        host = torch.from_numpy(tokenize(seq)[None]).pin_memory()
        dev = host.to(self.model.device, non_blocking=True)
        N.note_transfer(h2d=host.nbytes)
        return seq, host, dev

    def generate(self, prompt: str, n_tokens: int = 256, *, greedy: bool = False, gamma: int | None = None,
                 seed: int = 0, temperature: float = 1.0, top_k: int = 4) -> GenerateResult:
        import torch

        from evspark_b200.specdec.block.loop import speculative_generate

        from evspark_b200.specdec.block.driver import prefill

        g = int(gamma) if gamma else self.gamma
        self._nd.capture_reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        seq, host_ids, ids = self._ids_pinned(prompt)
        L = int(ids.shape[1])
        # prefill the prompt (all but its last token, the first anchor) into the kept decode state,
        # with the drafter capturing its context, as speculative_generate does with a fresh state
        ip = self._decode_state(L + int(n_tokens) + g + 2)
        self._nd.capture_begin()
        prefill(self.model, ids[:, :-1], ip)
        self._nd.capture_commit(L - 1)
        spec = speculative_generate(self.model, self._nd, host_ids, int(n_tokens), g, greedy=greedy,
                                    rng=np.random.default_rng(seed), temperature=temperature, top_k=top_k,
                                    rollback="slice", timing=False, inference_params_dict=ip)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ks = [int(r.k) for r in spec.rounds_log]
        out = np.asarray(spec.emitted_ids)
        return GenerateResult(text=ids_to_text(out), ids=out, mode="greedy" if greedy else "sampling",
                              speculative=True, n_tokens=int(n_tokens), wall_s=wall,
                              tok_s=float(n_tokens / wall) if wall > 0 else float("nan"),
                              mean_tau=float(np.mean(ks) + 1.0) if ks else None, n_rounds=len(ks),
                              extra={"gamma": g, "seed": seed, "prompt_bp": len(seq), "rounds": spec.rounds_log})

    def generate_native(self, prompt: str, n_tokens: int = 256, *, greedy: bool = False, seed: int = 0,
                        temperature: float = 1.0, top_k: int = 4) -> GenerateResult:
        import torch

        from evspark_b200.specdec.block.loop import native_greedy_reference, native_sample_reference

        seq, ids = self._ids(prompt)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if greedy:
            out, ip, _ = native_greedy_reference(self.model, ids, int(n_tokens))
            ip.close()
        else:
            out = native_sample_reference(self.model, ids, int(n_tokens), np.random.default_rng(seed),
                                          temperature=temperature, top_k=top_k)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        out = np.asarray(out)
        return GenerateResult(text=ids_to_text(out), ids=out, mode="greedy" if greedy else "sampling",
                              speculative=False, n_tokens=int(n_tokens), wall_s=wall,
                              tok_s=float(n_tokens / wall) if wall > 0 else float("nan"),
                              extra={"seed": seed, "prompt_bp": len(seq)})

    def close(self) -> None:
        if self._state is not None:
            self._state.close()
            self._state = None
        if self._nd is not None:
            self._nd.close()
            self._nd = None
        if self.model is not None:
            self.model.close()

    def __enter__(self) -> "EvSpark":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
