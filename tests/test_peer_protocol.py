"""The peer exchange protocol of the sharded searches, as a host model.

Each rank is a thread that runs the searches' sequence of arena writes and
exchanges in order (a GPU stream runs them in order too).  An exchange is
what the kernel does: store this rank's epoch into its word of the slot's
flag line in every arena, wait until every word of its own arena's line is
at least the epoch, then read the other ranks' sections.  Sections are
tagged with the epoch that wrote them, and every read must see its own
epoch -- neither an older value (read too early) nor a newer one (the owner
overwrote it before the reader was done).  Random delays between steps
explore the interleavings; a search without a threshold exchange (shard
sizes too small for the shared sample) is mixed in, which is the case the
two list sections exist for.
"""
import random
import threading

import pytest

SLOT_MAXIMA, SLOT_THRESHOLD, SLOT_LISTS, SLOT_PROBE = 0, 1, 2, 3


class Model:
    def __init__(self, world):
        self.world = world
        self.flags = [[[0] * world for _ in range(4)] for _ in range(world)]  # [arena][slot][writer]
        self.arena = [dict() for _ in range(world)]                            # [rank][section] = epoch
        self.cv = threading.Condition()
        self.errors = []

    def write(self, r, section, epoch):
        with self.cv:
            self.arena[r][section] = epoch

    def exchange(self, r, slot, epoch, section, rng, own=True):
        with self.cv:
            for p in range(self.world):                  # signal: st.release.sys into every arena
                self.flags[p][slot][r] = epoch
            self.cv.notify_all()
            ok = self.cv.wait_for(lambda: all(f >= epoch for f in self.flags[r][slot]), timeout=10)
            if not ok:
                self.errors.append(f"rank {r}: wait for slot {slot} epoch {epoch} ran out")
                return
        delay(rng)                                       # the copy takes a while
        with self.cv:
            for p in range(self.world):
                if p == r and not own:
                    continue
                got = self.arena[p].get(section)
                if got != epoch:
                    self.errors.append(f"rank {r} read {section} of rank {p}: epoch {got}, wanted {epoch}")


def delay(rng):
    if rng.random() < 0.5:
        threading.Event().wait(rng.random() * 2e-4)


def flat_rank(m, r, steps, with_threshold, seed):
    """ShardedSearch.search with the peer transport, `steps` searches."""
    rng = random.Random(seed * 1009 + r)
    for e in range(1, steps + 1):
        delay(rng)
        if with_threshold(e):
            m.write(r, "maxima", e)                       # sample pass into the arena
            m.exchange(r, SLOT_MAXIMA, e, "maxima", rng)  # owner reads every rank's maxima
            delay(rng)
            m.write(r, "thr", e)                          # this rank's slice of thresholds
            m.exchange(r, SLOT_THRESHOLD, e, "thr", rng, own=False)
        delay(rng)
        name = "lists%d" % (e & 1)
        m.write(r, name, e)                               # packed lists
        m.exchange(r, SLOT_LISTS, e, name, rng)


def ivf_rank(m, r, steps, seed):
    """ShardedIVFSearch.search with the peer transport."""
    rng = random.Random(seed * 2003 + r)
    for e in range(1, steps + 1):
        delay(rng)
        m.write(r, "probe", e)                            # this rank's slice of the probe table
        m.exchange(r, SLOT_PROBE, e, "probe", rng, own=False)
        delay(rng)
        name = "lists%d" % (e & 1)
        m.write(r, name, e)
        m.exchange(r, SLOT_LISTS, e, name, rng)


def run(world, target, *args):
    m = Model(world)
    ts = [threading.Thread(target=target, args=(m, r) + args) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in ts)
    return m.errors


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("seed", range(3))
def test_flat_exchanges_never_read_a_stale_or_overwritten_section(world, seed):
    # threshold exchanges on most searches, none on every third (the lists
    # are then exchanged twice in a row)
    errors = run(world, flat_rank, 60, lambda e: e % 3 != 0, seed)
    assert not errors, errors[:5]


@pytest.mark.parametrize("world", [2, 8])
def test_ivf_exchanges_never_read_a_stale_or_overwritten_section(world):
    errors = run(world, ivf_rank, 60, 7)
    assert not errors, errors[:5]


def test_one_list_section_would_be_overwritten():
    """The model catches the hazard the second list section removes: with
    one section and no threshold exchange between searches, a rank that
    runs ahead rewrites its lists while another still reads them."""

    def single_section_rank(m, r, steps, seed):
        rng = random.Random(seed * 31 + r)
        for e in range(1, steps + 1):
            m.write(r, "lists", e)
            if r == 0:
                # rank 0 copies slowly; rank 1 runs ahead into the next search
                m.exchange(r, SLOT_LISTS, e, "lists_slow", rng)
            else:
                m.exchange(r, SLOT_LISTS, e, "lists", rng)

    class SlowRead(Model):
        def exchange(self, r, slot, epoch, section, rng, own=True):
            if section != "lists_slow":
                return super().exchange(r, slot, epoch, section, rng, own)
            with self.cv:
                for p in range(self.world):
                    self.flags[p][slot][r] = epoch
                self.cv.notify_all()
                self.cv.wait_for(lambda: all(f >= epoch for f in self.flags[r][slot]), timeout=10)
            threading.Event().wait(0.02)  # the other rank writes its next lists meanwhile
            with self.cv:
                got = self.arena[1].get("lists")
                if got != epoch:
                    self.errors.append(f"rank 0 read lists of rank 1: epoch {got}, wanted {epoch}")

    m = SlowRead(2)
    ts = [threading.Thread(target=single_section_rank, args=(m, r, 3, 0)) for r in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert any("wanted 1" in e for e in m.errors), m.errors
