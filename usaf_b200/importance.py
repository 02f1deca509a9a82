"""Dense importance scores (drop-in for usaf/importance.py).

``ImportanceScorer.compute_scores`` keeps the reference's behaviour
(usaf/importance.py:24-111): the model in eval mode, every parameter whose
name matches none of ``skip_patterns`` made trainable, one forward/backward
of ``outputs.loss`` per batch (1-D inputs get a batch dimension; at most
``max_batches`` batches when > 0), ``|grad|`` summed in fp32 per parameter,
a batch that raises an out-of-memory ``RuntimeError`` skipped (20 in a row
end the pass, other errors propagate), every scored parameter frozen again
at the end, and zeros for parameters that never received a gradient.

Differences that follow from the device design: the sums stay on the
parameters' device (the reference copies every gradient to the CPU), and
int4 expert tensors attached with :func:`usaf_b200.qwen3moe.attach_int4_experts`
-- which are not parameters here -- are scored through the ``_grad_capture``
protocol with a :class:`usaf_b200.moe_loader.DenseAbsGradStore` (|dW| of every
expert from the tensor-core dense-gradient kernel), under the names the
reference's expert parameters have (``<experts>.gate_up_proj`` /
``<experts>.down_proj``).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from .moe_loader import DenseAbsGradStore

MAX_CONSECUTIVE_SKIPS = 20   # usaf/importance.py:41


class ImportanceScorer:
    DEFAULT_SKIP: Tuple[str, ...] = ("embed_tokens", "lm_head")

    def __init__(self, model: torch.nn.Module, device: torch.device, dtype: torch.dtype,
                 context_length: int = 2048, skip_patterns: Optional[Tuple[str, ...]] = None):
        self.model = model
        self.device = device
        self.dtype = dtype
        self.context_length = context_length
        self.skip_patterns = skip_patterns or self.DEFAULT_SKIP

    def _int4_experts(self):
        return {n: m for n, m in self.model.named_modules() if getattr(m, "_usaf_int4", None) is not None}

    def compute_scores(self, dataloader, max_batches: int = 0) -> Dict[str, torch.Tensor]:
        self.model.eval()
        grad_accum: Dict[str, torch.Tensor] = {}
        param_name_map = {}
        for name, param in self.model.named_parameters():
            skip = any(pat in name for pat in self.skip_patterns)
            param.requires_grad = not skip
            if not skip:
                param_name_map[name] = param
        experts = self._int4_experts()
        shapes = {}
        for n, m in experts.items():
            gu, dn = m._usaf_int4
            for which, p in (("gate_up_proj", gu), ("down_proj", dn)):
                full = f"{n}.{which}"
                if not any(pat in full for pat in self.skip_patterns):
                    shapes[full] = p.shape
        store = DenseAbsGradStore(shapes)
        saved = {n: m.__dict__.get("_grad_capture") for n, m in experts.items()}
        for n, m in experts.items():
            m._grad_capture = (store, n)
        batches_processed = 0
        consecutive_skips = 0
        try:
            for batch in dataloader:
                if max_batches > 0 and batches_processed >= max_batches:
                    break
                input_ids = batch["input_ids"].to(self.device)
                labels = batch["labels"].to(self.device)
                if input_ids.dim() == 1:
                    input_ids = input_ids.unsqueeze(0)
                    labels = labels.unsqueeze(0)
                try:
                    try:
                        outputs = self.model(input_ids=input_ids, labels=labels)
                    except TypeError:
                        outputs = self.model(input_ids=input_ids, labels=labels, pixel_values=None)
                    loss = outputs.loss
                    if loss is not None:
                        self.model.zero_grad(set_to_none=True)
                        loss.backward()
                        for name, param in param_name_map.items():
                            if param.grad is not None:
                                g = param.grad.detach().float().abs_()
                                if name in grad_accum:
                                    grad_accum[name] += g
                                else:
                                    grad_accum[name] = g
                    batches_processed += 1
                    consecutive_skips = 0
                except RuntimeError as e:
                    if "memory" in str(e).lower() or "allocate" in str(e).lower():
                        consecutive_skips += 1
                        if consecutive_skips >= MAX_CONSECUTIVE_SKIPS:
                            break
                    else:
                        raise
                finally:
                    self.model.zero_grad(set_to_none=True)
                    del input_ids, labels
        finally:
            for n, m in experts.items():
                if saved[n] is None:
                    m.__dict__.pop("_grad_capture", None)
                else:
                    m._grad_capture = saved[n]
            for name, param in param_name_map.items():
                param.requires_grad = False

        scores: Dict[str, torch.Tensor] = {}
        for name, param in self.model.named_parameters():
            if name in grad_accum:
                scores[name] = grad_accum[name]
            else:
                scores[name] = torch.zeros(param.shape, dtype=torch.float32, device=param.device)
        for full, shape in shapes.items():
            dev = experts[full.rsplit(".", 1)[0]]._usaf_int4[0].device
            scores[full] = store.scores.get(full, None)
            if scores[full] is None:
                scores[full] = torch.zeros(tuple(shape), dtype=torch.float32, device=dev)
        return scores

    def save_scores(self, scores: Dict[str, torch.Tensor], path: str) -> None:
        """usaf/importance.py:106-108 (fp16 copies, CPU tensors in the file)."""
        torch.save({k: v.detach().half().cpu() for k, v in scores.items()}, path)

    @staticmethod
    def load_scores(path: str) -> Dict[str, torch.Tensor]:
        return torch.load(path, map_location="cpu", weights_only=True)
