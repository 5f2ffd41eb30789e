"""Expert residency (glc_moe_set_expert_slots): every layer's routed experts in
pinned host memory and a few HBM slots, filled as the routing selects them --
the GPU slot cache of GpuFirstExpertStageWorker (GpuFirstExpertStageWorker.cs:
144-151, 344-407).

Outputs, expert ids and combine weights equal the fully resident layer's bit
for bit on the decode and the batched path; the hit / transfer / prefetch
counters follow a model of the slot policy run beside it (key (layer, expert),
the least recently used slot out, never one the same call uses; layer 0's
first experts staged when it is loaded); a call routing to more distinct
experts than there are slots is refused.
"""
import numpy as np
import pytest

from test_gpu_parity import make_layer

pytestmark = pytest.mark.gpu

DECODE, BATCHED = 4, 8
GLC_ERR_UNSUPPORTED, GLC_ERR_STATE = -4, -8


class SlotModel:
    class Full(Exception):
        pass

    def __init__(self, n):
        self.key, self.used, self.clock = [None] * n, [0] * n, 0
        self.hits = self.transfers = self.prefetches = 0

    def _ensure(self, key, stamp):
        if key in self.key:
            self.used[self.key.index(key)] = stamp
            return False
        free = [i for i in range(len(self.key)) if self.used[i] < stamp]
        if not free:
            raise SlotModel.Full()
        v = min(free, key=lambda i: (self.used[i], i))
        self.key[v], self.used[v] = key, stamp
        return True

    def load(self, layer, E):
        for i, k in enumerate(self.key):
            if k is not None and k[0] == layer:
                self.key[i], self.used[i] = None, 0
        if layer == 0:
            self.clock += 1
            for e in range(min(len(self.key), E)):
                self._ensure((0, e), self.clock)

    def call(self, layer, ids):
        self.clock += 1
        for e in ids:
            if self._ensure((layer, int(e)), self.clock):
                self.transfers += 1
            else:
                self.hits += 1

    def prefetch(self, layer, ids):
        self.clock += 1
        for e in ids:
            try:
                if self._ensure((layer, int(e)), self.clock):
                    self.prefetches += 1
            except SlotModel.Full:
                break

    def counters(self):
        return {"slots": len(self.key), "hits": self.hits, "transfers": self.transfers,
                "prefetches": self.prefetches}


def _load(w, l, L):
    w.load_layer(l, L["gate"], L["up"], L["down"], L["router"])


def test_paged_experts_equal_resident_layer_and_count_like_the_slot_cache(cuda, glc, oracle):
    D, F, E, k, slots = 512, 1024, 8, 2, 4
    Ls = [make_layer(oracle, 4100 + l, D, F, E, k) for l in range(2)]
    full = glc.GpuExpertStageWorker(D, F, E, k, num_layers=2, max_tokens=4)
    paged = glc.GpuExpertStageWorker(D, F, E, k, num_layers=2, max_tokens=4, expert_slots=slots)
    model = SlotModel(slots)
    for l in range(2):
        _load(full, l, Ls[l])
        _load(paged, l, Ls[l])
        model.load(l, E)
    assert paged.expert_residency() == model.counters()
    calls = [(0, 1, 3 | DECODE), (1, 1, 3 | DECODE), (1, 2, 3 | BATCHED), (0, 1, 1 | DECODE), (0, 2, 3 | DECODE),
             (1, 1, 3 | DECODE), (0, 2, 3 | BATCHED), (1, 2, 2 | DECODE)]
    for i, (layer, T, flags) in enumerate(calls):
        x = oracle.fill_normal(4200 + i, 1, 1.0, T * D).reshape(T, D)
        fo, fids, fw = full.forward(layer, x, flags)
        po, pids, pw = paged.forward(layer, x, flags)
        assert np.array_equal(pids, fids) and np.array_equal(pw, fw), i
        assert np.array_equal(po, fo), (i, float(np.abs(po - fo).max()))
        model.call(layer, fids.reshape(-1))
        assert paged.expert_residency() == model.counters(), i
    # lookahead prefetch: the next call's experts staged ahead are hits
    x = oracle.fill_normal(4300, 1, 1.0, D).reshape(1, D)
    _, fids, _ = full.forward(1, x, 3 | DECODE)
    paged.prefetch_experts(1, fids.reshape(-1))
    model.prefetch(1, fids.reshape(-1))
    assert paged.expert_residency() == model.counters()
    po, pids, _ = paged.forward(1, x, 3 | DECODE)
    model.call(1, fids.reshape(-1))
    c = paged.expert_residency()
    assert c == model.counters() and np.array_equal(pids, fids)
    assert c["prefetches"] >= 1 or c["hits"] >= 2
    # a reloaded layer's slots are dropped (its experts may have changed)
    L2 = make_layer(oracle, 4400, D, F, E, k)
    _load(full, 1, L2)
    _load(paged, 1, L2)
    model.load(1, E)
    fo, fids, _ = full.forward(1, x, 3 | DECODE)
    po, pids, _ = paged.forward(1, x, 3 | DECODE)
    model.call(1, fids.reshape(-1))
    assert np.array_equal(po, fo) and paged.expert_residency() == model.counters()
    paged.poll_error()
    full.dispose()
    paged.dispose()


def test_more_distinct_experts_than_slots_is_refused(cuda, glc, oracle):
    D, F, E, k = 512, 1024, 8, 2
    L = make_layer(oracle, 4500, D, F, E, k)
    paged = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=4, expert_slots=2)
    _load(paged, 0, L)
    ids = None
    for seed in range(4600, 4700):  # four tokens that route to at least three distinct experts
        x = oracle.fill_normal(seed, 1, 1.0, 4 * D).reshape(4, D)
        _, ids, _ = oracle.moe_forward(L, x, 3)
        if len(set(np.asarray(ids).reshape(-1).tolist())) > 2:
            break
    with pytest.raises(glc.GlcError) as e:
        paged.forward(0, x, 3 | DECODE)
    assert e.value.status == GLC_ERR_UNSUPPORTED
    assert paged.expert_residency()["slots"] == 2
    paged.dispose()


def test_expert_slots_arguments(cuda, glc, oracle):
    D, F, E, k = 512, 1024, 8, 2
    L = make_layer(oracle, 4800, D, F, E, k)
    w = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=2, expert_slots=64)  # clamped to E
    assert w.expert_residency()["slots"] == E
    w.dispose()
    w = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=2)
    assert w.expert_residency() == {"slots": E, "hits": 0, "transfers": 0, "prefetches": 0}
    w.prefetch_experts(0, [1, 2])  # every expert resident: nothing to do
    _load(w, 0, L)
    # slots are set before the first layer is loaded
    assert glc.lib().glc_moe_set_expert_slots(w._handle(), 2) == GLC_ERR_STATE
    w.dispose()
