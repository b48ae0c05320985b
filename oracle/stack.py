"""The GLM decode stack of configuration 5 on the CPU oracle (greedy-token checker).

TEST INFRASTRUCTURE ONLY: used by tests/ and by bench.py's stack leg to check greedy
tokens and time the CPU baseline; the product stack is diskmule_b200.stack.GlmStack,
whose host-side bytes (embedding rows, norms, expert blobs) this class reads.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


class OracleStack:
    """The same stack on the CPU oracle: per step the embedding row, per layer
    h += glm_block(rms_norm(h)), the final norm, the head and argmax
    (src/glm52/cpu.rs:476-518, :711-778, :912-924; src/cpu.rs:276-292)."""

    def __init__(self, stack, threads: int = 8):
        self.O, self.stack, self.threads = O, stack, threads
        self.layers = [stack.host_layer(l) for l in range(stack.n_layers)]
        self.head = stack.head_spec.host()
        self.selections = []  # per step, per layer: selected experts in order

    def step(self, token: int) -> int:
        O, st = self.O, self.stack
        h = st.embed_row(token).copy()
        sel = []
        for l, w in enumerate(self.layers):
            rc, n = O.glm_rms_norm(h, st.norms[l], st.epsilon)
            assert rc == O.OK
            rc, y, idx, _ = O.glm_moe(w, n[None, :], threads=self.threads)
            assert rc == O.OK, rc
            sel.append(idx[0].tolist())
            h = (h + y[0]).astype(np.float32)
        rc, n = O.glm_rms_norm(h, st.out_norm, st.epsilon)
        rc, logits = O.glm_matvec(O.BF16, st.vocab, st.H, self.head, n, threads=self.threads)
        assert rc == O.OK
        rc, best = O.argmax(logits)
        assert rc == O.OK
        self.selections.append(sel)
        self.last_hidden = h
        return int(best)

    def decode(self, first_token: int, steps: int):
        out, tok = [], first_token
        for _ in range(steps):
            tok = self.step(tok)
            out.append(tok)
        return out
