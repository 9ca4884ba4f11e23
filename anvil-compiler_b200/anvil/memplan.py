"""Static memory planner for a lowered launch chain: liveness over the op order, then offsets that let a buffer
reuse the bytes of buffers dead before it is defined.

Follows the reference planner anvil/memplan.py (liveness :96-153, assign_offsets :64-81, check_disjoint :84-93)
with the unit changed from tiny-gpu words to device bytes and an alignment (256 B, so every arena buffer can be a
TMA base and a 16-byte vector address):

    a buffer is live on the closed interval [def, last use] of op indices; inputs are defined at -1 (copied in
    before the first launch), graph outputs (and every value when keep="all") stay live to n (read back after
    the last launch); two buffers whose intervals intersect never overlap in memory. Offsets are greedy: largest
    first (ties: earliest start, then name), each at the lowest aligned offset that fits between the already
    placed buffers it conflicts with.

The const region is not planned here: constants are packed once per model (anvil.runtime.program).
"""
from __future__ import annotations

from dataclasses import dataclass, field

ALIGN = 256


class MemoryPlanError(ValueError):
    """The planned job does not fit (anvil/memplan.py:27-28)."""


@dataclass(frozen=True)
class Buf:
    sym: str
    size: int                   # bytes
    start: int                  # first op index where live (-1: before the first launch)
    end: int                    # last op index where live (n: read after the last launch)
    kind: str = "act"           # "input" | "act" | "output"

    def overlaps(self, o: "Buf") -> bool:
        return self.start <= o.end and o.start <= self.end


@dataclass
class MemPlan:
    addresses: dict                             # sym -> arena byte offset
    bufs: dict                                  # sym -> Buf
    arena: int = 0                              # arena bytes
    const_bytes: int = 0
    guard: int = 0                              # guarded plan: bytes of canary after every buffer (no reuse)

    def inside(self) -> "np.ndarray":
        """Boolean mask over the arena's bytes: True where some planned buffer lives (the bytes a correct launch
        chain may change); everything else is alignment gap or guard."""
        import numpy as np
        m = np.zeros(self.arena, dtype=bool)
        for s, b in self.bufs.items():
            a = self.addresses[s]
            m[a:a + b.size] = True
        return m

    @property
    def unshared(self) -> int:
        """Arena bytes a bump allocator (no reuse) would need."""
        return sum(_align(b.size) for b in self.bufs.values())

    @property
    def footprint(self) -> int:
        return self.arena + self.const_bytes

    def report(self) -> str:
        g = f"; guarded, {self.guard} canary bytes after every buffer" if self.guard else ""
        return (f"footprint {self.footprint} bytes (consts {self.const_bytes}, activations {self.arena}; "
                f"activations without reuse {self.unshared}{g})")


def _align(n: int, a: int = ALIGN) -> int:
    return -(-int(n) // a) * a


def assign_offsets(bufs, align: int = ALIGN) -> tuple[dict, int]:
    """({sym: offset}, arena bytes) with no two simultaneously-live buffers overlapping."""
    order = sorted(bufs, key=lambda b: (-b.size, b.start, b.sym))
    placed: list[tuple[int, Buf]] = []
    out, top = {}, 0
    for b in order:
        size = _align(b.size, align)
        busy = sorted((o, o + _align(p.size, align)) for o, p in placed if p.overlaps(b) and p.size)
        off = 0
        for lo, hi in busy:
            if off + size <= lo:
                break
            off = max(off, _align(hi, align))
        out[b.sym] = off
        placed.append((off, b))
        top = max(top, off + size)
    return out, top


def assign_guarded(bufs, guard: int, align: int = ALIGN) -> tuple[dict, int]:
    """({sym: offset}, arena bytes) for a debug run: every buffer its own bytes (no reuse), each followed by at
    least `guard` bytes that belong to no buffer, so a store past any buffer's end lands in a guard region."""
    out, top = {}, 0
    for b in sorted(bufs, key=lambda b: (b.start, b.sym)):
        out[b.sym] = top
        top = _align(top + b.size + guard, align)
    return out, top


def check_disjoint(bufs, addresses) -> list:
    """Pairs of simultaneously-live buffers whose byte ranges intersect (empty for a sound plan)."""
    bad, bl = [], list(bufs)
    for i, a in enumerate(bl):
        for b in bl[i + 1:]:
            if a.size and b.size and a.overlaps(b):
                x, y = addresses[a.sym], addresses[b.sym]
                if x < y + b.size and y < x + a.size:
                    bad.append((a.sym, b.sym))
    return bad


def liveness(n_ops: int, sizes: dict, defs: dict, uses: dict, inputs, outputs, keep: str = "outputs") -> dict:
    """sym -> Buf. `defs` sym -> defining op index, `uses` sym -> [op indices reading it]."""
    if keep not in ("outputs", "all"):
        raise ValueError(f"keep must be 'outputs' or 'all', not {keep!r}")
    out = {}
    ins, outs = set(inputs), set(outputs)
    for s, size in sizes.items():
        start = -1 if s in ins else defs[s]
        last = max([start] + list(uses.get(s, ())))
        kind = "input" if s in ins else "act"
        if s in outs or keep == "all":
            last = n_ops
            if kind == "act":
                kind = "output"
        out[s] = Buf(s, int(size), start, last, kind)
    return out


def plan(n_ops: int, sizes: dict, defs: dict, uses: dict, inputs, outputs, keep="outputs", const_bytes=0,
         max_bytes: int | None = None, guard: int = 0) -> MemPlan:
    """The liveness plan; with `guard` > 0 the debug layout of assign_guarded instead (stray-write checks)."""
    bufs = liveness(n_ops, sizes, defs, uses, inputs, outputs, keep)
    offs, arena = assign_guarded(bufs.values(), guard) if guard else assign_offsets(bufs.values())
    mp = MemPlan(offs, bufs, arena, const_bytes, guard)
    if max_bytes is not None and mp.footprint > max_bytes:
        raise MemoryPlanError(f"plan needs {mp.footprint} bytes > {max_bytes}: " + mp.report())
    bad = check_disjoint(bufs.values(), offs)
    if bad:                                           # unreachable unless assign_offsets is broken
        raise MemoryPlanError(f"live buffers overlap: {bad[:4]}")
    return mp
