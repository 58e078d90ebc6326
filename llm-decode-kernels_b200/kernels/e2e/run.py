"""End-to-end decode timing on a Qwen2 runner (reference kernels/e2e/run.py, without the HF
download, perplexity and chat prompts, which need the network).

- `GraphDecoder`: one greedy decode step (forward + argmax + position bump) captured in a CUDA
  graph and replayed per token (reference run.py:58-111), for batch 1 or more.
- `decode_speed`: median tok/s over repeats (reference run.py:114-122).
- `prefill_speed`, `layers_only_ms`: reference run.py:142-201.
- `step_host`: the public per-token API of a server loop - the token comes from pinned host memory,
  the graph runs, the next token is read back to the host.
- `greedy_parity`: the reference's parity figures (run.py:289-303) between two runners - max |logit
  diff| and the first greedy divergence - for batch-1 synthetic prompts.
"""

from __future__ import annotations

import statistics

import torch

from kernels.bench.harness import capture
from kernels.e2e.model import QwenRunner


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


class GraphDecoder:
    """Captures one greedy decode step (forward + argmax + bookkeeping) in a CUDA graph."""

    def __init__(self, runner: QwenRunner):
        self.r = runner
        dev = runner.embed.device
        B = runner.batch
        self.tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.out = torch.zeros(B, runner.max_len, dtype=torch.long, device=dev)
        self.graph = None
        self.host_tok = torch.zeros(B, 1, dtype=torch.long).pin_memory()
        self.host_next = torch.zeros(B, 1, dtype=torch.long).pin_memory()

    def _step(self):
        logits = self.r.forward(self.tok, self.pos)
        nxt = self.r.greedy(logits)
        self.out.index_copy_(1, self.pos, nxt.view(-1, 1))
        self.tok.copy_(nxt.view(-1, 1))
        self.pos.add_(1)

    def prefill(self, ids: torch.Tensor):
        """ids [B, P] on the device. Fills the cache, sets the first generated token."""
        P = ids.shape[1]
        logits = self.r.forward(ids, torch.arange(P, device=ids.device))
        self.tok.copy_(self.r.greedy(logits).view(-1, 1))
        self.pos.fill_(P)
        self.out.zero_()
        self.out[:, P - 1] = self.tok.view(-1)  # position P-1 holds the first new token
        return P

    def capture(self, ids):
        # warm up outside the graph (kernel choices, library loads), then reset the state
        self.prefill(ids)
        self._step()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.prefill(ids)
        self.graph, _ = capture(self._step)
        torch.cuda.synchronize()

    def generate(self, ids, steps: int) -> tuple[list, float]:
        P = self.prefill(ids)
        torch.cuda.synchronize()
        start, end = _events()
        start.record()
        for _ in range(steps):
            self.graph.replay()
        end.record()
        torch.cuda.synchronize()
        tokens = self.out[:, P - 1: P - 1 + steps + 1].tolist()
        return tokens, start.elapsed_time(end) / 1e3

    def step_host(self, token_host: torch.Tensor) -> torch.Tensor:
        """One token through the public API from host memory: copy the token in (pinned host ->
        device), replay the step, copy the next token out (device -> pinned host) and wait for it."""
        self.host_tok.copy_(token_host)
        self.tok.copy_(self.host_tok, non_blocking=True)
        self.graph.replay()
        self.host_next.copy_(self.tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.host_next


def decode_speed(runner, ids, steps: int, repeats: int = 3) -> dict:
    dec = GraphDecoder(runner)
    dec.capture(ids)
    rates = []
    for _ in range(repeats):
        _, sec = dec.generate(ids, steps)
        rates.append(steps * runner.batch / sec)
    return {"tok_s": statistics.median(rates), "tok_s_min": min(rates), "tok_s_max": max(rates),
            "ms_per_step": 1e3 * runner.batch / statistics.median(rates), "steps": steps,
            "batch": runner.batch}


def prefill_speed(runner, T: int, repeats: int = 5) -> dict:
    dev = runner.embed.device
    ids = torch.randint(0, runner.embed.shape[0], (runner.batch, T), device=dev)
    pos = torch.arange(T, device=dev)
    for _ in range(2):
        runner.forward(ids, pos)
    torch.cuda.synchronize()
    graph, _ = capture(lambda: runner.forward(ids, pos))
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(repeats):
        start, end = _events()
        start.record()
        graph.replay()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) / 1e3)
    del graph
    t = statistics.median(times)
    return {"T": T, "ms": t * 1e3, "tok_s": runner.batch * T / t}


def layers_only_ms(runner, M: int = 1) -> float:
    """Graph time of the swapped ops of one decode step: per layer the qkv, o, gate_up(+act) and
    down projections and the two fused add+norms; no attention, embedding or lm_head
    (reference run.py:166-201)."""
    be, eps = runner.backend, runner.eps
    dev = runner.embed.device
    H = runner.embed.shape[1]
    x = torch.randn(1, M, H, device=dev, dtype=torch.float16)
    res = torch.randn_like(x)
    nq, hd = runner.n_heads, runner.head_dim

    def step():
        h, r = be.norm(x, runner.layers[0].ln1, eps, residual=res)
        for L in runner.layers:
            qkv = be.linear(h, L.qkv)
            o = be.linear(qkv[..., : nq * hd].contiguous(), L.o)
            h, r = be.norm(o, L.ln2, eps, residual=r)
            h = be.linear(be.gate_up_act(h, L.gate_up), L.down)
            h, r = be.norm(h, L.ln1, eps, residual=r)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graph, _ = capture(step)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(7):
        start, end = _events()
        start.record()
        for _ in range(10):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) / 10)
    del graph
    return statistics.median(times)


@torch.no_grad()
def greedy_parity(runner: QwenRunner, ref: QwenRunner, ids: torch.Tensor, steps: int = 32) -> dict:
    """Greedy decode of `steps` tokens after the prompt `ids` [1, T] by `runner` and by `ref`, each on
    its own KV cache (eager forward steps), fed the same tokens until they disagree. Reports what
    the reference's parity check reports (kernels/e2e/run.py:289-303): the max |logit diff| over the
    compared positions and the index of the first greedy divergence (`steps` if none; greedy streams
    part for good after one near-tie, so where they part is the figure, not a match fraction), plus
    the reference's top-2 logit margin at that position (a divergence needs a logit error of at
    least half of it) and the largest |reference logit| (for relative tolerances)."""
    T = ids.shape[1]
    dev = ids.device
    pos = torch.arange(T, device=dev)
    la = runner.forward(ids, pos)[:, -1].float()
    lb = ref.forward(ids, pos)[:, -1].float()
    diff = (la - lb).abs().max().item()
    ref_abs = lb.abs().max().item()
    toks: list[int] = []
    first, margin = steps, None
    for i in range(steps):
        a, b = int(la[0].argmax()), int(lb[0].argmax())
        if a != b:
            top2 = lb[0].topk(2).values
            first, margin = i, (top2[0] - top2[1]).item()
            break
        toks.append(b)
        if i + 1 == steps:
            break
        tok = torch.tensor([[b]], device=dev)
        p = torch.tensor([T + i], device=dev)
        la = runner.forward(tok, p)[:, -1].float()
        lb = ref.forward(tok, p)[:, -1].float()
        diff = max(diff, (la - lb).abs().max().item())
        ref_abs = max(ref_abs, lb.abs().max().item())
    return {"max_abs_logit_diff": diff, "max_abs_ref_logit": ref_abs, "first_divergence": first,
            "compared_tokens": steps, "ref_margin_at_divergence": margin, "tokens": toks}
