"""Decision heads: a backbone's option-scoring readout instead of the LM head.

A Decision 2.0 package is a Qwen3 backbone plus `decision_head.safetensors`.
The prompt lists the options (for AI.IF / AI.SCORE: No, then Yes) and the
head reads, per answer, the row that ends each option and the prompt's last
row, all after the final RMSNorm. Each option row and the last row pass
through their own LayerNorm; the option's score is

    score_i = <key(c_i), query(q)> / sqrt(d) + scalar . gelu(cmlp(c_i) + qmlp(q))

with c_i = LN_c(option row i), q = LN_q(last row), d the head width.

Split of the work: the GPU turns every read row into its four projections
([key(c) | cmlp(c) | query(q) | qmlp(q)], fp32, two GEMMs over the
readout rows of a pass), so only 4d floats per row cross to the host; the
per-answer combination above (a dot product and a d-wide GELU per option)
runs on the host when the answer's rows arrive. `scores` is the whole head
in one torch statement, the reference the split is tested against.

Reference: quail/backends/quail/executor/readout.py:491-552 (DecisionHead),
:633-728 (DecisionRows and the filter / score / classify readouts);
models/decision2.py (the backbone's tensor names).
"""

from __future__ import annotations

import math

import numpy as np
import torch

TENSORS = ("candidate_norm.weight", "candidate_norm.bias", "query_norm.weight", "query_norm.bias",
           "key.weight", "query.weight", "candidate_mlp.weight", "candidate_mlp.bias", "query_mlp.weight",
           "scalar.weight")
PREFIX = "decision_head."


def random_decision_head(hidden: int, dim: int, gen: torch.Generator, device="cpu") -> dict[str, torch.Tensor]:
    """Random-init head tensors under `decision_head.<name>` (fp32)."""
    def rnd(*shape, std):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std
    s = hidden ** -0.5
    t = {
        "candidate_norm.weight": 1.0 + rnd(hidden, std=0.02), "candidate_norm.bias": rnd(hidden, std=0.02),
        "query_norm.weight": 1.0 + rnd(hidden, std=0.02), "query_norm.bias": rnd(hidden, std=0.02),
        "key.weight": rnd(dim, hidden, std=s), "query.weight": rnd(dim, hidden, std=s),
        "candidate_mlp.weight": rnd(dim, hidden, std=s), "candidate_mlp.bias": rnd(dim, std=0.02),
        "query_mlp.weight": rnd(dim, hidden, std=s), "scalar.weight": rnd(1, dim, std=dim ** -0.5),
    }
    return {PREFIX + k: v for k, v in t.items()}


def head_tensors(ckpt: dict) -> dict[str, torch.Tensor]:
    """The head's tensors of a checkpoint dict, by their names in decision_head.safetensors."""
    got = {k[len(PREFIX):]: v for k, v in ckpt.items() if k.startswith(PREFIX)}
    missing = set(TENSORS) - got.keys()
    if missing:
        raise ValueError(f"the decision head is missing {sorted(missing)}")
    unknown = got.keys() - set(TENSORS)
    if unknown:
        raise ValueError(f"the decision head does not use {sorted(unknown)}")
    return got


class DecisionHead:
    def __init__(self, tensors: dict[str, torch.Tensor], device):
        w = {k: v.to(device=device, dtype=torch.float32).contiguous() for k, v in tensors.items()}
        self.w = w
        self.dim = w["key.weight"].shape[0]
        self.hidden = w["key.weight"].shape[1]
        # candidate side [key | cmlp] and query side [query | qmlp], one GEMM each
        self.wc = torch.cat([w["key.weight"], w["candidate_mlp.weight"]]).contiguous()
        self.bc = torch.cat([torch.zeros(self.dim, device=device), w["candidate_mlp.bias"]]).contiguous()
        self.wq = torch.cat([w["query.weight"], w["query_mlp.weight"]]).contiguous()
        self.scalar = w["scalar.weight"][0].detach().cpu().numpy().astype(np.float64)

    @property
    def width(self) -> int:
        """Floats per readout row of `features`."""
        return 4 * self.dim

    def features(self, normed: torch.Tensor) -> torch.Tensor:
        """[R, hidden] final-normed rows -> [R, 4d] fp32: [key(c) | cmlp(c) | query(q) | qmlp(q)]."""
        w = self.w
        x = normed.float()
        H = x.shape[-1]
        c = torch.nn.functional.layer_norm(x, (H,), w["candidate_norm.weight"], w["candidate_norm.bias"])
        q = torch.nn.functional.layer_norm(x, (H,), w["query_norm.weight"], w["query_norm.bias"])
        return torch.cat([torch.addmm(self.bc, c, self.wc.t()), q @ self.wq.t()], dim=1)

    def combine(self, rows) -> np.ndarray:
        """Rows of one answer (options first, the last row last) -> one float score per option."""
        a = np.asarray(rows, dtype=np.float64).reshape(-1, self.width)
        d = self.dim
        opt, last = a[:-1], a[-1]
        key, cmlp = opt[:, :d], opt[:, d:2 * d]
        query, qmlp = last[2 * d:3 * d], last[3 * d:]
        bilinear = key @ query / math.sqrt(d)
        z = cmlp + qmlp[None, :]
        gelu = 0.5 * z * (1.0 + _erf(z / math.sqrt(2.0)))
        return bilinear + gelu @ self.scalar

    def scores(self, options: torch.Tensor, last: torch.Tensor) -> torch.Tensor:
        """(prompts, options, hidden), (prompts, hidden) -> (prompts, options): the head in one statement."""
        F, w = torch.nn.functional, self.w
        H = options.shape[-1]
        o = F.layer_norm(options.float(), (H,), w["candidate_norm.weight"], w["candidate_norm.bias"])
        q = F.layer_norm(last.float(), (H,), w["query_norm.weight"], w["query_norm.bias"])
        bil = (F.linear(o, w["key.weight"]) * F.linear(q, w["query.weight"])[:, None, :]).sum(-1)
        mlp = F.linear(F.gelu(F.linear(o, w["candidate_mlp.weight"], w["candidate_mlp.bias"])
                              + F.linear(q, w["query_mlp.weight"])[:, None, :]), w["scalar.weight"]).squeeze(-1)
        return bil / math.sqrt(self.dim) + mlp


def _erf(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf
    return erf(x)
