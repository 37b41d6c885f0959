"""dspark::spec::run on device (tools/dspark/src/spec.rs:25-283): greedy speculative decode
of a target ``DeviceModel`` with a ``DeviceDraft``.

The loop is the reference's: the target processes the prompt's positions 0..P-2 and holds
the last prompt token back as the first anchor; every round the draft proposes a block at
pos0 (decode_block), the target verifies [anchor, proposals] at pos0.. in one batch
(spk_model_verify), the longest matching prefix k plus the target's own token are
committed, the target rolls back to pos0 + k + 1, and the draft's injected features of
the committed rows are encoded from the target's layer-input captures. The reference
re-encodes every committed position each round (spec.rs:188-189); a position's encoding
depends only on its captures, so encoding each committed row once is the same computation.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SpecResult:
    generated: list = field(default_factory=list)
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    proposals: list = field(default_factory=list)   # per round
    targets: list = field(default_factory=list)     # per round


def prepare(target, draft) -> None:
    """Model::enable_capture with the draft's target layers (spec.rs:141)."""
    target.enable_capture(draft.cfg.target_layers)
    draft.use_target_head(target)


def run(target, draft, ids: list, gen: int, n_max: int | None = None, acceptor=None) -> SpecResult:
    """spec.rs::run: returns the generated ids and the round statistics. ``acceptor``
    (optional, for synthetic-acceptance benchmarks) maps (round, proposals, target ids) to
    the committed prefix length instead of the match rule."""
    cfg = draft.cfg
    if len(ids) < 2:
        raise ValueError("spec needs at least two prompt ids")
    n_draft = min(n_max or cfg.draft_max(), cfg.draft_max())
    if n_draft == 0:
        raise ValueError("n_max is zero for this draft")
    i_beg = cfg.i_beg()
    pos0 = len(ids) - 1
    for p, t in enumerate(ids[:pos0]):
        target.forward(t, p, want_logits=False)
    caps, stride = target.captures()
    draft.encode_features(caps, stride, 0, pos0)
    anchor = ids[pos0]
    out = SpecResult()
    embed, vocab = target.embed_dev.data_ptr(), target.cfg.vocab
    while len(out.generated) < gen:
        block, _, _ = draft.decode_block(embed, vocab, anchor, pos0, n_draft)
        proposals = block[i_beg:]
        if len(proposals) != n_draft:
            raise RuntimeError(f"draft produced {len(proposals)} proposals for n_draft {n_draft}")
        tgt, _ = target.verify([anchor] + proposals, pos0)
        k = 0
        while k < n_draft and tgt[k] == proposals[k]:
            k += 1
        if acceptor is not None:
            k = acceptor(out.rounds, proposals, tgt)
        out.generated += proposals[:k] + [tgt[k]]
        out.drafted += n_draft
        out.accepted += k
        out.rounds += 1
        out.proposals.append(proposals)
        out.targets.append(tgt)
        target.rollback(pos0 + k + 1)
        draft.encode_features(caps, stride, pos0, pos0 + k + 1)
        pos0 += k + 1
        anchor = tgt[k]
    out.generated = out.generated[:gen]
    return out
