"""Thinking-token budgets (`SamplingParams.thinking_token_budget`) over the engine's greedy tokens.

A reasoning model thinks between its start and end markers, whose token IDs vLLM's reasoning
config names (`--reasoning-parser`). Once a request has emitted `budget` tokens inside a thinking
section without ending it, its next tokens are the end marker's tokens, one a step, whatever the
model chose; a section the model ends itself, or a new one it starts, is tracked the same way.

The engine picks tokens on the device, so a forced token replaces the engine's token when the
runner reads the step, and the next step feeds it from the host. A request with a budget therefore
has its tokens read as each step is issued. With speculative drafts, the accepted tokens after a
replaced one are dropped (their rows were verified against the token that was replaced) and the
request's cached positions are rolled back by as many.
"""

from __future__ import annotations


class Budget:
    def __init__(self, budget: int, start, end):
        if budget < 0:
            raise ValueError(f"thinking_token_budget: {budget}, not negative")
        if not end:
            raise ValueError("thinking_token_budget: the reasoning config names no end marker tokens")
        self.budget, self.start, self.end = int(budget), tuple(int(t) for t in start), tuple(int(t) for t in end)
        self.reset(())

    def reset(self, tokens, prompt: int | None = None) -> None:
        """Derives the state from a request's tokens so far, of which the first `prompt` (all by
        default) are its prompt: a prompt may open a thinking section (a chat template that ends
        with the start marker), and only emitted tokens count against the budget."""
        # Without a start marker a request thinks from its first token.
        self.thinking, self.spent, self.forced, self.recent = not self.start, 0, 0, []
        tokens = [int(t) for t in tokens]
        prompt = len(tokens) if prompt is None else prompt
        for t in tokens[:prompt]:
            self._advance(t)
        self.spent = 0
        for t in tokens[prompt:]:
            self._advance(t)

    def _ends_with(self, marker) -> bool:
        return bool(marker) and tuple(self.recent[-len(marker):]) == marker

    def _advance(self, token: int) -> None:
        self.recent = (self.recent + [token])[-max(len(self.start), len(self.end)):]
        if self.thinking:
            if self._ends_with(self.end):
                self.thinking, self.forced = False, 0
            else:
                self.spent += 1
        elif self._ends_with(self.start):
            self.thinking, self.spent = True, 0

    def choose(self, token: int) -> int:
        """The token the request emits where the engine chose `token`."""
        if self.thinking and (self.forced or self.spent >= self.budget):
            token = self.end[self.forced]
            self.forced += 1
        self._advance(int(token))
        return int(token)


def apply(budget: Budget, tokens: list[int]) -> list[int]:
    """A step's tokens after the budget: the first replaced token ends the list."""
    out = []
    for t in tokens:
        c = budget.choose(t)
        out.append(c)
        if c != t:
            break
    return out
