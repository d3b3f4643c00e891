"""Stateful property test of the serving request slots (host side, no
GPU): any interleaving of admissions, one-token appends and releases keeps
the accounting exact -- every live request owns exactly its pages, no page
has two owners, free + live slots equal the admission capacity, a released
lease is stale for good -- and every append ages only finished pages into
the INT8 history, as the reference's request_slots.py requires."""

from __future__ import annotations

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import settings, strategies as st  # noqa: E402
from hypothesis.stateful import (RuleBasedStateMachine, initialize, invariant,  # noqa: E402
                                 precondition, rule)

from pagegauge_b200.serving import PAGE, Policy, RequestSlots, exact_slot, partition  # noqa: E402

POLICY = Policy(prefix_pages=1, suffix_pages=2, tail_pages=3)
CAPACITY = 3


class SlotsMachine(RuleBasedStateMachine):
    @initialize()
    def start(self):
        self.slots = RequestSlots(CAPACITY, POLICY)
        self.next_page = 0
        self.next_id = 0
        self.live = {}        # request id -> lease
        self.released = []    # stale leases

    def _fresh_pages(self, n):
        pages = list(range(self.next_page, self.next_page + n))
        self.next_page += n
        return pages

    @precondition(lambda self: len(self.live) < CAPACITY)
    @rule(prompt=st.integers(7 * PAGE, 12 * PAGE))
    def admit(self, prompt):
        rid = f"r{self.next_id}"
        self.next_id += 1
        lease = self.slots.admit(rid, prompt, self._fresh_pages(-(-prompt // PAGE)))
        self.live[rid] = lease

    @precondition(lambda self: len(self.live) == CAPACITY)
    @rule()
    def admit_over_capacity(self):
        with pytest.raises(MemoryError):
            self.slots.admit("extra", 8 * PAGE, self._fresh_pages(8))

    @precondition(lambda self: self.live)
    @rule(data=st.data(), tokens=st.integers(1, 20))
    def append(self, data, tokens):
        rid = data.draw(st.sampled_from(sorted(self.live)))
        lease = self.live[rid]
        for _ in range(tokens):
            state = self.slots.state(lease)
            pos = state.current_tokens
            need = -(-(pos + 1) // PAGE)
            pages = list(state.physical_pages) + self._fresh_pages(need - len(state.physical_pages))
            out = self.slots.append(lease, pos, pages)
            # Only finished pages age into the history.
            assert all(p < (pos + 1) // PAGE for p in out["new_history_pages"])
            assert out["closed_page"] == (pos // PAGE if (pos + 1) % PAGE == 0 else None)

    @precondition(lambda self: self.live)
    @rule(data=st.data())
    def release(self, data):
        rid = data.draw(st.sampled_from(sorted(self.live)))
        lease = self.live.pop(rid)
        self.slots.release(lease)
        self.released.append(lease)

    @precondition(lambda self: self.released)
    @rule(data=st.data())
    def stale_lease_rejected(self, data):
        lease = data.draw(st.sampled_from(self.released))
        with pytest.raises(ValueError):
            self.slots.state(lease)

    @invariant()
    def accounting(self):
        if not hasattr(self, "slots"):
            return
        owned = {}
        for rid, lease in self.live.items():
            state = self.slots.state(lease)
            for p in state.physical_pages:
                assert p not in owned
                owned[p] = lease
        assert owned == self.slots.page_owner
        assert len(self.slots.free) + len(self.live) == CAPACITY
        assert sorted(self.slots.free + [l.slot for l in self.live.values()]) == list(range(CAPACITY))
        # Exact pages of every live request sit in distinct sidecar slots of
        # its own lease slot.
        for lease in self.live.values():
            state = self.slots.state(lease)
            part = partition(state.prompt_tokens, state.current_tokens, POLICY)
            sl = [exact_slot(p, state.prompt_tokens, lease.slot, POLICY) for p in part["exact"]]
            assert len(set(sl)) == len(sl)
            base = lease.slot * POLICY.storage_pages
            assert all(base <= s < base + POLICY.storage_pages for s in sl)


TestSlots = SlotsMachine.TestCase
TestSlots.settings = settings(max_examples=60, stateful_step_count=25, deadline=None)
