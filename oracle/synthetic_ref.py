"""numpy restatement of the reference's synthetic single-layer decoder.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``SyntheticDecodeRunner`` (reference ``src/inferkernellab/decode.py``):
the weights of ``_make_weights`` (``:261-279``), the projections of
``_project_query`` / ``_project_kv`` (``:292-304``) and one decode step of
``_decode`` (``:465-493``): the query token is the last prompt token at step 0
and the previously generated token after that; the KV cache holds every
earlier token (prompt + generated) at its logical position; attention runs over
``prompt_len + step`` tokens; ``out_proj`` then ``lm_head`` give the logits and
the next token is their argmax.

The decoder is evaluated *teacher-forced*: given the generated tokens of a run,
``decode_logits`` returns the float32 logits the reference math produces at every
step for that token history.
"""

from __future__ import annotations

import numpy as np

from .paged_ref import dense_decode_attention


def make_weights(vocab_size: int, num_heads: int, num_kv_heads: int, head_dim: int, seed: int):
    """The reference's seeded weights as float32 numpy arrays (decode.py:261-279).

    Uses torch's CPU generator exactly as the reference does (normal draws in
    the same order and scales); the caller rounds them to the model dtype.
    """
    import torch

    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    hidden = num_heads * head_dim
    kv = num_kv_heads * head_dim

    def w(shape, scale):
        return (torch.randn(shape, generator=gen, dtype=torch.float32) * scale).numpy()

    hs = hidden ** -0.5
    return {
        "embedding": w((vocab_size, hidden), 0.02),
        "q_proj": w((hidden, hidden), hs),
        "k_proj": w((kv, hidden), hs),
        "v_proj": w((kv, hidden), hs),
        "out_proj": w((hidden, hidden), hs),
        "lm_head": w((vocab_size, hidden), hs),
    }


def decode_logits(weights: dict, prompts, generated, num_heads: int, num_kv_heads: int,
                  head_dim: int) -> list[np.ndarray]:
    """Float32 logits ``[R, vocab]`` of every decode step for a token history.

    ``weights``: float32 arrays (already rounded to the model dtype if the run
    was fp16/bf16).  ``generated[r]`` = the tokens request ``r`` produced.
    """
    emb = weights["embedding"].astype(np.float32)
    wq, wk, wv = (weights[k].astype(np.float32) for k in ("q_proj", "k_proj", "v_proj"))
    wo, wl = weights["out_proj"].astype(np.float32), weights["lm_head"].astype(np.float32)
    steps = len(generated[0])
    out = []
    for step in range(steps):
        rows = []
        for prompt, gen in zip(prompts, generated):
            history = list(prompt) + list(gen[:step])
            current = prompt[-1] if step == 0 else gen[step - 1]
            hidden_ctx = emb[np.asarray(history, dtype=np.int64)]
            key = (hidden_ctx @ wk.T).reshape(len(history), num_kv_heads, head_dim)
            value = (hidden_ctx @ wv.T).reshape(len(history), num_kv_heads, head_dim)
            query = (emb[current] @ wq.T).reshape(num_heads, head_dim)
            attn = dense_decode_attention(query, key, value)
            hidden = attn.reshape(-1) @ wo.T
            rows.append(hidden @ wl.T)
        out.append(np.stack(rows).astype(np.float32))
    return out
