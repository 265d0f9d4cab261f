"""The coordinator's side of a layer pipeline, as rakkan-mesh's Service runs
it (internal/llm/generate.go:415-595, runStage 616-719): the prompt through
every stage in one request, then one token per pass, each stage's output the
next one's input, and greedy sampling at the end. A stage whose node fails
moves to another node, and its cache is rebuilt by replaying every input
the stage has received so far, which the coordinator keeps
(generate.go:616-719).

A stage here is anything with forward(xs, pos) -> xs' (rows of dim floats
at positions pos, pos+1, ...) and close(): in this package an rk.Stage (or
a PipelineRank's layers) on a GPU; the placement callback opens one for a
layer span on a node, as Service.place does (generate.go:600-614). The
reference's trust layer (witness nodes, generate.go:636-672, 721-755) and
its network placement are not part of this path.
"""
import numpy as np

MAX_ATTEMPTS = 3  # failovers per pass before the error is returned (generate.go:697)


class StageError(RuntimeError):
    pass


class PlannedStage:
    """planned (generate.go): a span of layers [from_, to) on a node, and
    the inputs it has received, one activation row per position (the
    reference keeps them as bytes with per-position ends)."""

    def __init__(self, from_, to, node, conn):
        self.from_, self.to = from_, to
        self.node, self.conn = node, conn
        self.inputs = []  # one float32 row per position received
        self.failovers = 0


def run_stage(st, xs, pos, place, others=()):
    """runStage (generate.go:616-719): xs [count][dim] at positions pos.. in,
    the stage's output out. A pass from an earlier position first rewinds
    what the stage received from there on; a position past the stage's
    inputs is an error. If the node fails, place(st, exclude) opens the
    stage on another node (it sets st.node and st.conn), the inputs so far
    are replayed into it, and the pass is retried, at most MAX_ATTEMPTS
    times."""
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    if xs.ndim == 1:
        xs = xs[None, :]
    if pos < len(st.inputs):
        del st.inputs[pos:]  # the rewind (generate.go:620-628)
    if pos != len(st.inputs):
        raise StageError(f"layers {st.from_}..{st.to}: position {pos} after {len(st.inputs)}")
    attempt = 0
    while True:
        try:
            out = st.conn.forward(xs.copy(), pos)
        except Exception as err:  # the node failed: move the stage
            if attempt >= MAX_ATTEMPTS:
                raise StageError(f"layers {st.from_}..{st.to}: {err}") from err
            attempt += 1
            try:
                st.conn.close()
            except Exception:
                pass
            exclude = {st.node} | {o.node for o in others if o is not st}
            if not place(st, exclude):
                # Doubling up on a node already in the pipeline beats failing.
                if not place(st, {st.node}):
                    raise StageError(f"layers {st.from_}..{st.to}: no node to move the stage to") from err
            if pos > 0:
                try:
                    st.conn.forward(np.stack(st.inputs), 0)  # replay (generate.go:711-715)
                except Exception:
                    continue
            st.failovers += 1
            continue
        st.inputs.extend(np.array(r, copy=True) for r in xs)
        return np.ascontiguousarray(out, dtype=np.float32).reshape(xs.shape)


def generate(stages, embed, logits_of, prompt, max_tokens, place, stop=(), seq_len=None):
    """Service.Generate's loop without a draft (generate.go:511-586):
    embed(tokens) -> rows, logits_of(row) -> logits; the prompt through
    every stage in one pass, then one token per pass, the next token the
    first strict maximum of the logits (Sampler.Sample at temperature 0,
    sample.go:45-53). Returns (new tokens, stats).

    seq_len is the stages' context (positions their caches hold). As in
    generate.go:442-450, a prompt that fills it is refused, and max_tokens
    is clamped to the positions left (max_tokens <= 0: all of them), so a
    run ends at the context instead of passing a position the stages
    cannot hold (which would read as a node failure)."""
    tokens = list(prompt)
    if not tokens:
        raise ValueError("empty prompt")
    if seq_len is not None:
        if len(tokens) >= seq_len:
            raise ValueError(f"prompt of {len(tokens)} tokens fills the context of {seq_len}")
        left = seq_len - len(tokens)
        max_tokens = min(max_tokens, left) if max_tokens > 0 else left
    stats = {"passes": 0, "tokens": 0, "failovers": 0}
    pos, out = 0, []
    xs = embed(tokens)
    while stats["tokens"] < max_tokens:
        stats["passes"] += 1
        for st in stages:
            xs = run_stage(st, xs, pos, place, stages)
        lg = np.asarray(logits_of(xs[-1]), dtype=np.float32)
        nxt = first_max(lg)
        if nxt in stop:
            break
        tokens.append(nxt)
        out.append(nxt)
        stats["tokens"] += 1
        pos = len(tokens) - 1
        xs = embed(tokens[pos:])
    stats["failovers"] = sum(st.failovers for st in stages)
    return out, stats


def first_max(v):
    """argmax (sample.go:45-53): the first index of the strict maximum; a NaN
    never compares greater, and a NaN at index 0 stays the answer."""
    v = np.asarray(v, dtype=np.float32)
    if v.size == 0 or np.isnan(v[0]):
        return 0
    return int(np.argmax(np.where(np.isnan(v), -np.inf, v)))
