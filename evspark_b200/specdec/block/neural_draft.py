"""Neural drafter decode adapter (mirror of evspark/specdec/block/neural_draft.py:262-456).

``NeuralDraftModel`` keeps the reference's loop protocol — ``capture_begin`` /
``capture_commit(n_keep)`` / ``capture_buffer_len`` / ``capture_reset`` and
``propose_block(anchor, γ', greedy, rng, ...) -> (tokens[γ'], q_rows[γ', V], conf[γ'])`` — but
the hidden-state capture is native: the target forward writes the injection layers' outputs
into the state's capture ring, rollback trims it for free (the ring is indexed by absolute
position and the context is the last ``min(ctx_window, len)`` consumed positions), and drafting
is one device call.  Only committed (consumed) positions are ever visible, exactly the
reference's "rejected suffix is dropped at commit" rule.

RNG: in sampling mode the serial head consumes exactly γ' uniforms (one per draft position,
neural_draft.py:233-250), pre-drawn here in order; greedy drafting consumes none.
"""

from __future__ import annotations

import numpy as np
import torch

from evspark_b200.drafter import SCHEME_LAYERS, DeviceDrafter, layer_index, load_checkpoint


class NeuralDraftModel:
    def __init__(self, model, drafter: DeviceDrafter, layer_names: tuple[str, ...], *, ctx_maxlen: int | None = None):
        self.model = model
        self.drafter = drafter
        self.layer_names = tuple(layer_names)
        self.gamma = int(drafter.gamma)
        want = tuple(layer_index(n) for n in self.layer_names)
        have = tuple(model.capture_layers[: len(want)])
        if want != have:
            raise ValueError(f"target model captures blocks {model.capture_layers}, drafter needs {want}: build the "
                             "TargetModel with capture_layers matching the drafter's injection layers")
        self.maxlen = int(ctx_maxlen or drafter.ctx_window)
        self.total_committed = 0
        self._armed = False

    @classmethod
    def from_checkpoint(cls, model, ckpt_path: str, *, device="cuda:0") -> "NeuralDraftModel":
        drafter, layers, meta = load_checkpoint(ckpt_path, model.cfg.d_model, device=device)
        inst = cls(model, drafter, layers)
        inst.ckpt_meta = meta
        return inst

    # -- loop protocol ------------------------------------------------------
    def capture_begin(self) -> None:
        self._armed = True

    def capture_commit(self, n_keep: int, batch_idx: int = 0) -> None:
        if not self._armed:
            raise RuntimeError("capture_commit needs a preceding capture_begin")
        self._armed = False
        self.total_committed += int(n_keep)

    def capture_buffer_len(self) -> int:
        return int(self.total_committed)

    def capture_reset(self) -> None:
        self.total_committed = 0
        self._armed = False

    def _check_gamma(self, gamma: int) -> None:
        if int(gamma) > self.gamma:
            raise ValueError(f"decode γ={gamma} > drafter training γ={self.gamma}: only decode γ <= training γ "
                             f"(the pos table has {self.gamma} rows)")

    def propose_device(self, anchor: torch.Tensor, gamma: int, greedy: bool, rng, *, temperature=1.0, top_k=4,
                       inference_params_dict=None):
        """Device-resident proposal for the loop: returns device (tokens [1,γ], q fp64 [1,γ,V], conf)."""
        self._check_gamma(gamma)
        ip = inference_params_dict
        if ip is None:
            raise ValueError("the device drafter reads its context from inference_params_dict")
        u = None
        if not greedy:
            u = torch.as_tensor(rng.random(int(gamma)), device=self.drafter.device)[None]
        toks, q, conf, _ = self.drafter.propose(ip, anchor.reshape(1), int(gamma), greedy, temperature=temperature,
                                                top_k=top_k, uniforms=u)
        return toks, q, conf

    def propose_blocks_device(self, anchor_id: int, gamma: int, greedy: bool, rng, n_candidates: int, *,
                              temperature=1.0, top_k=4, inference_params_dict=None):
        """``n_candidates`` drafts from one anchor (neural_draft.py:366-446), on rows 0..B-1 of a state
        expanded to B identical rows.  Sampling: i.i.d. candidates, γ uniforms each, in candidate order.
        Greedy: the B most probable first tokens of q_0 (ties: lower id), each followed by argmax steps.
        Returns device (tokens [B, γ], q fp64 [B, γ, V], conf [B, γ])."""
        self._check_gamma(gamma)
        ip = inference_params_dict
        if ip is None:
            raise ValueError("the device drafter reads its context from inference_params_dict")
        B = int(n_candidates)
        if B < 1:
            raise ValueError(f"n_candidates must be >= 1, got {B}")
        dev = self.drafter.device
        anchors = torch.full((B,), int(anchor_id), dtype=torch.int64, device=dev)
        if greedy:
            _, _, _, U = self.drafter.propose(ip, anchors[:1], int(gamma), True, want_U=True)
            q0 = torch.softmax((U[0, 0] + self.drafter.weights["markov"][int(anchor_id)]).float(), dim=-1)
            top = torch.sort(-q0, stable=True).indices[:B]
            forced = torch.full((B, int(gamma)), -1, dtype=torch.int64, device=dev)
            forced[:, 0] = top
            toks, q, conf, _ = self.drafter.propose(ip, anchors, int(gamma), True, forced=forced)
        else:
            u = torch.as_tensor(np.stack([rng.random(int(gamma)) for _ in range(B)]), device=dev)
            toks, q, conf, _ = self.drafter.propose(ip, anchors, int(gamma), False, temperature=temperature,
                                                    top_k=top_k, uniforms=u)
        return toks, q, conf

    @torch.no_grad()
    def propose_blocks(self, anchor_id: int, gamma: int, greedy: bool, rng: np.random.Generator, n_candidates: int,
                       *, temperature: float = 1.0, top_k: int | None = 4, inference_params_dict=None, **_kw):
        """Host view of ``propose_blocks_device``: (tokens [B, γ], q_rows [B, γ, V], confs [B, γ])."""
        toks, q, conf = self.propose_blocks_device(anchor_id, gamma, greedy, rng, n_candidates,
                                                   temperature=temperature, top_k=top_k,
                                                   inference_params_dict=inference_params_dict)
        return toks.cpu().numpy(), q.cpu().numpy(), conf.double().cpu().numpy()

    @torch.no_grad()
    def propose_block(self, anchor_id: int, gamma: int, greedy: bool, rng: np.random.Generator, *,
                      temperature: float = 1.0, top_k: int | None = 4, inference_params_dict=None, **_kw):
        anchor = torch.tensor([int(anchor_id)], dtype=torch.int64, device=self.drafter.device)
        toks, q, conf = self.propose_device(anchor, gamma, greedy, rng, temperature=temperature, top_k=top_k,
                                            inference_params_dict=inference_params_dict)
        return toks[0].cpu().numpy(), q[0].cpu().numpy(), conf[0].double().cpu().numpy()

    def close(self) -> None:
        self.drafter.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


__all__ = ["NeuralDraftModel", "SCHEME_LAYERS"]
