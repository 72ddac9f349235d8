"""The barrier protocols of the chunk-attention kernel (lingbot-world-v2_b200/csrc/attn.cu, chunk_attn_kernel) and of
the persistent GEMMs (csrc/gemm_bf16.cu gemm_bf16_kernel: two TMEM accumulators; csrc/gemm_mx.cu gemm_mx_kernel:
one) run in the discrete-event model of tests/protocol_model.py under random TMA / MMA latencies, delayed commit
arrivals, ragged tiles and random O rescales: no aliased parity wait, no deadlock, and the hazards below hold
where the kernels rely on them.

Attention:

The programs restate the kernel's synchronisation, step for step:
  producer   Q once; per key tile j: wait k_empty[j % 2] (use j / 2), load K; wait v_empty, load V
  watcher    K(0) landed; per tile j: V(j) landed -> arrive p_ready[0][0]; K(j + 1) landed -> arrive p_ready[0][1];
             then wait for both phases of tile j to complete (so its next arrivals cannot land in them)
  issuer     S_0 = Q_0 K_0^T (and S_1 with two query tiles), commit s_full; commit k_empty[0]; per tile j:
             wait p_ready[0][0] (P_0 keys 0..63 and V(j)) -> P_0 V (keys 0..63); wait p_ready[0][1] (P_0 keys
             64..127 and K(j + 1)) -> P_0 V (keys 64..127); next S_0, commit s_full[0]; then the same P_1 V for the
             second tile; commit v_empty; next S_1, commit s_full[1]; commit k_empty; finally commit o_done
  softmax i  per tile: wait s_full[i]; P over S; without a rescale and on a full tile it arrives p_ready[i][0]
             once keys 0..63 of P are written, else after the rescale of O; then p_ready[i][1]
Hazards: S is complete when read; P V starts only after every softmax warp wrote its part of P and V landed; the next
S only after K landed; P (j) is written only after the P V that read P (j - 1) completed; O is rescaled only while
no P V of that query tile runs; a K or V ring slot is refilled only after every MMA that read it completed; every
arrival lands in the phase it is meant for.

Persistent GEMM (one CTA's tiles t = 0, 1, ...):
  producer   per tile, per K stage: wait empty[s] (its previous use), load A and B into slot s
  issuer     per tile: wait tempty[acc] (the epilogue has released that accumulator), per K stage wait full[s],
             MMAs into the accumulator, commit empty[s]; then commit tfull[acc]; acc alternates (two accumulators)
             or stays 0 (one)
  epilogue   each of the 8 warps per tile: wait tfull[acc], read its rows of the accumulator, arrive tempty[acc]
Hazards: the accumulator is read only after every MMA of its tile completed, and is written by the next tile's
MMAs only after all 8 warps read it; a ring slot is refilled only after the MMAs that read it completed.

Sequence-parallel K/V exchange (csrc/peer.cu lbw_sp_kv_stage / lbw_sp_kv_gather, driven by block.py
_self_attention), per rank and exchange e:
  main stream    the block's kernels (which write this rank's rows of the destination chunk); stage: wait
                 done[me][p] >= e - 1 from every peer, copy this rank's rows into its staging buffer, record an event;
                 the gated attention (whose destination-chunk tiles wait for gathered >= e); wait for the comm stream
  comm stream    wait that event; write ready[p][me] = e in every peer's buffer; wait ready[me][p] >= e; start the
                 pulls; join them; write done[p][me] = e in every peer's buffer; write gathered[me] = e
  pull streams   (one per peer) copy the peer's staging buffer into its rows of the destination chunk
Hazards: a staging buffer is rewritten only after every peer's pull of it finished, and is pulled only once it
holds the exchange's rows; the attention reads the destination chunk only when every rank's rows of this exchange
have landed."""
import random

import pytest

from protocol_model import Bar, Flag, Model


def attention_v1(m, n_tiles, two, rescale_p, ragged_p, watcher_phase_wait=True):
    nq = 2 if two else 1
    q_full = Bar("q_full")
    k_full, k_empty = [Bar(f"k_full{s}") for s in range(2)], [Bar(f"k_empty{s}") for s in range(2)]
    v_full, v_empty = [Bar(f"v_full{s}") for s in range(2)], [Bar(f"v_empty{s}") for s in range(2)]
    s_full = [Bar(f"s_full{i}") for i in range(2)]
    # 4 softmax warps per warpgroup; query tile 0's two barriers also take the watcher's arrival
    p_ready = [[Bar(f"p_ready{i}{h}", 4 + (i == 0)) for h in range(2)] for i in range(2)]
    o_done = Bar("o_done")
    MMA_S, MMA_PV = 512, 256                     # 128 x 128 x 128 S; P V over 64 keys
    p_written = {}                               # (query tile, key tile, half) -> softmax warps that wrote it

    def producer():
        yield ("tma", q_full, ("Q",))
        for j in range(n_tiles):
            s = j & 1
            yield ("wait", k_empty[s], j >> 1)
            if j >= 2:
                for i in range(nq):
                    assert m.complete(("S", i, j - 2)), ("K slot refilled while read", j)
            yield ("tma", k_full[s], ("K", j))
            yield ("wait", v_empty[s], j >> 1)
            if j >= 2:
                for i in range(nq):
                    for h in range(2):
                        assert m.complete(("PV", i, h, j - 2)), ("V slot refilled while read", j)
            yield ("tma", v_full[s], ("V", j))

    def watcher():
        yield ("wait", k_full[0], 1)             # every landing observed in order, K(0) first
        for j in range(n_tiles):
            yield ("wait", v_full[j & 1], (j >> 1) + 1)
            assert p_ready[0][0].k == j, ("watcher arrival in another phase", j)
            yield ("arrive", p_ready[0][0])
            if j + 1 < n_tiles:
                yield ("wait", k_full[(j + 1) & 1], ((j + 1) >> 1) + 1)
            assert p_ready[0][1].k == j, ("watcher arrival in another phase", j)
            yield ("arrive", p_ready[0][1])
            if watcher_phase_wait:
                yield ("wait", p_ready[0][0], j + 1)
                yield ("wait", p_ready[0][1], j + 1)

    def issuer():
        yield ("wait", q_full, 1)
        yield ("wait", k_full[0], 1)
        for i in range(nq):
            yield ("mma", ("S", i, 0), MMA_S)
            yield ("commit", s_full[i])
        yield ("commit", k_empty[0])
        for j in range(n_tiles):
            s, more, s1 = j & 1, j + 1 < n_tiles, (j + 1) & 1
            yield ("wait", p_ready[0][0], j + 1)
            assert ("V", j) in m.loaded and p_written.get((0, j, 0), 0) == 4, ("P V before V / P", 0, j)
            yield ("mma", ("PV", 0, 0, j), MMA_PV)
            yield ("wait", p_ready[0][1], j + 1)
            assert (not more or ("K", j + 1) in m.loaded) and p_written.get((0, j, 1), 0) == 4, ("S before K", j)
            yield ("mma", ("PV", 0, 1, j), MMA_PV)
            if more:
                yield ("mma", ("S", 0, j + 1), MMA_S)
                yield ("commit", s_full[0])
            if two:
                yield ("wait", p_ready[1][0], j + 1)
                assert p_written.get((1, j, 0), 0) == 4, ("P V before P", 1, j)
                yield ("mma", ("PV", 1, 0, j), MMA_PV)
                yield ("wait", p_ready[1][1], j + 1)
                assert p_written.get((1, j, 1), 0) == 4, ("P V before P", 1, j)
                yield ("mma", ("PV", 1, 1, j), MMA_PV)
            yield ("commit", v_empty[s])
            if more:
                if two:
                    yield ("mma", ("S", 1, j + 1), MMA_S)
                    yield ("commit", s_full[1])
                yield ("commit", k_empty[s1])
        yield ("commit", o_done)

    def release(wg, j, h):
        for _ in range(4):
            p_written[(wg, j, h)] = p_written.get((wg, j, h), 0) + 1
            assert p_ready[wg][h].k == j, ("softmax arrival in another phase", wg, j, h)
            yield ("arrive", p_ready[wg][h])

    def softmax(wg):
        for j in range(n_tiles):
            yield ("wait", s_full[wg], j + 1)
            assert m.complete(("S", wg, j)), ("S read before complete", wg, j)
            if j >= 1:
                for h in range(2):
                    assert m.complete(("PV", wg, h, j - 1)), ("P overwritten while read", wg, j)
            rescale = j > 0 and m.rng.random() < rescale_p
            full = m.rng.random() >= ragged_p
            # each half of the softmax from much shorter to much longer than the other tile's MMAs
            yield ("work", m.rng.uniform(150, 1300))
            if full and not rescale:
                yield from release(wg, j, 0)
            yield ("work", m.rng.uniform(150, 1300))
            if rescale:
                for tag in m.issued:
                    if tag[0] == "PV" and tag[1] == wg:
                        assert m.complete(tag), ("O rescaled while a P V runs", wg, j, tag)
                yield ("work", 300)
            if rescale or not full:
                yield from release(wg, j, 0)
            yield from release(wg, j, 1)
        yield ("wait", o_done, 1)
        for tag in m.issued:
            if tag[0] == "PV" and tag[1] == wg:
                assert m.complete(tag), ("epilogue before the last P V", wg)

    m.spawn(producer(), "producer")
    m.spawn(watcher(), "watcher")
    m.spawn(issuer(), "issuer")
    for wg in range(nq):
        m.spawn(softmax(wg), f"softmax{wg}")


@pytest.mark.parametrize("jitter", [0.0, 300.0, 3000.0])
def test_attention_protocol_random_schedules(jitter):
    for seed in range(400):
        rng = random.Random(seed)
        m = Model(seed, commit_jitter=jitter)
        attention_v1(m, n_tiles=rng.randint(1, 7), two=rng.random() < 0.7, rescale_p=rng.choice([0.0, 0.3, 1.0]),
                     ragged_p=rng.choice([0.0, 0.5]))
        m.run()


def test_model_catches_a_watcher_running_ahead():
    """Without its wait for each p_ready[0][h] phase, the watcher's arrival for the next key tile can land in the
    current phase (P V would start before every softmax warp has written P): the model must report it."""
    caught = 0
    for seed in range(50):
        m = Model(seed, tma_latency=(10.0, 20.0))
        attention_v1(m, n_tiles=5, two=True, rescale_p=0.0, ragged_p=0.0, watcher_phase_wait=False)
        try:
            m.run()
        except AssertionError:
            caught += 1
    assert caught > 0


def test_model_catches_a_wrong_phase():
    """A planted mistake in the model (the second query tile's issuer waits for the previous tile's P) must be
    reported."""
    def broken(m, n_tiles):
        b = Bar("p_ready")

        def softmax():
            for j in range(n_tiles):
                yield ("work", 10)
                yield ("arrive", b)

        def issuer():
            for j in range(n_tiles):
                yield ("work", 1000)
                yield ("wait", b, j)        # should be j + 1: passes on an older phase
        m.spawn(softmax(), "softmax")
        m.spawn(issuer(), "issuer")

    with pytest.raises(AssertionError):
        for seed in range(20):
            m = Model(seed)
            broken(m, 4)
            m.run()


def persistent_gemm(m, tiles, n_k, stages, n_acc, epi_warps=8):
    full, empty = [Bar(f"full{s}") for s in range(stages)], [Bar(f"empty{s}") for s in range(stages)]
    tfull, tempty = [Bar(f"tfull{a}") for a in range(n_acc)], [Bar(f"tempty{a}", epi_warps) for a in range(n_acc)]
    read = {}                      # tile -> number of epilogue warps that have read its accumulator

    def producer():
        use = [0] * stages
        s = 0
        for t in range(tiles):
            for kb in range(n_k):
                yield ("wait", empty[s], use[s])
                if use[s] > 0:
                    assert all(m.complete(tag) for tag in m.issued if tag[2] == (s, use[s] - 1)), "slot refilled"
                yield ("tma", full[s], ("AB", t, kb))
                use[s] += 1
                s = (s + 1) % stages

    def issuer():
        use = [0] * stages
        s = 0
        for t in range(tiles):
            acc = t % n_acc
            yield ("wait", tempty[acc], t // n_acc)
            if t >= n_acc:
                assert read.get(t - n_acc, 0) == epi_warps, ("accumulator overwritten while read", t)
            for kb in range(n_k):
                yield ("wait", full[s], use[s] + 1)
                yield ("mma", ("MMA", t, (s, use[s])), m.rng.uniform(100, 600))
                yield ("commit", empty[s])
                use[s] += 1
                s = (s + 1) % stages
            yield ("commit", tfull[acc])

    def epilogue(w):
        for t in range(tiles):
            acc = t % n_acc
            yield ("wait", tfull[acc], t // n_acc + 1)
            assert all(m.complete(tag) for tag in m.issued if tag[1] == t), ("accumulator read early", t)
            yield ("work", m.rng.uniform(50, 400))
            read[t] = read.get(t, 0) + 1
            yield ("arrive", tempty[acc])
            yield ("work", m.rng.uniform(0, 800))      # epilogue math after the release (one-accumulator kernel)

    m.spawn(producer(), "producer")
    m.spawn(issuer(), "issuer")
    for w in range(epi_warps):
        m.spawn(epilogue(w), f"epilogue{w}")


@pytest.mark.parametrize("n_acc,stages", [(2, 4), (2, 3), (1, 4), (1, 3)])
@pytest.mark.parametrize("jitter", [0.0, 2000.0])
def test_persistent_gemm_protocol_random_schedules(n_acc, stages, jitter):
    for seed in range(150):
        rng = random.Random(seed)
        m = Model(seed, commit_jitter=jitter)
        persistent_gemm(m, tiles=rng.randint(1, 6), n_k=rng.randint(1, 9), stages=stages, n_acc=n_acc)
        m.run()


def peer_exchange(m, world, epochs, skip_done_wait=False):
    ready = [[Flag(f"ready{x}{y}") for y in range(world)] for x in range(world)]   # in x's buffer, written by y
    done = [[Flag(f"done{x}{y}") for y in range(world)] for x in range(world)]
    gathered = [Flag(f"gathered{x}") for x in range(world)]
    ev_staged, ev_pull, ev_comm = ([Flag(f"{n}{x}") for x in range(world)] for n in ("staged", "pull", "comm"))
    ev_pulled = [[Flag(f"pulled{x}{y}") for y in range(world)] for x in range(world)]
    staging = [{"epoch": 0, "version": 0, "busy": False, "readers": 0} for _ in range(world)]
    dest = [[0] * world for _ in range(world)]      # exchange whose rows p sit in rank r's destination chunk
    peers = lambda r: [p for p in range(world) if p != r]

    def main(r):
        for e in range(1, epochs + 1):
            yield ("work", m.rng.uniform(100, 3000))       # the block's kernels; they write this rank's own rows
            dest[r][r] = e
            if e > 1 and not skip_done_wait:
                for p in peers(r):
                    yield ("waitge", done[r][p], e - 1)
            st = staging[r]

            def begin(st=st):
                assert st["readers"] == 0, "staging buffer rewritten while a peer pulls it"
                st["busy"], st["version"] = True, st["version"] + 1

            def end(st=st, e=e):
                st["busy"], st["epoch"] = False, e
            yield ("copy", begin, end, m.rng.uniform(50, 400))
            yield ("write", ev_staged[r], e)
            yield ("work", m.rng.uniform(0, 2000))          # attention over the leading chunks
            yield ("waitge", gathered[r], e)                # the gated tiles' poll
            assert all(dest[r][p] == e for p in range(world)), ("destination read before it landed", r, e)
            yield ("work", m.rng.uniform(0, 500))
            yield ("waitge", ev_comm[r], e)

    def comm(r):
        for e in range(1, epochs + 1):
            yield ("waitge", ev_staged[r], e)
            for p in peers(r):
                yield ("write", ready[p][r], e)
            for p in peers(r):
                yield ("waitge", ready[r][p], e)
            yield ("write", ev_pull[r], e)
            for p in peers(r):
                yield ("waitge", ev_pulled[r][p], e)
            for p in peers(r):
                yield ("write", done[p][r], e)
            yield ("write", gathered[r], e)
            yield ("write", ev_comm[r], e)

    def pull(r, p):
        for e in range(1, epochs + 1):
            yield ("waitge", ev_pull[r], e)
            st = staging[p]
            seen = {}

            def begin(st=st, e=e):
                assert not st["busy"] and st["epoch"] == e, ("pulled a staging buffer not holding the exchange", e)
                st["readers"] += 1
                seen["v"] = st["version"]

            def end(st=st, e=e):
                assert st["version"] == seen["v"], "staging buffer changed during a pull"
                st["readers"] -= 1
                dest[r][p] = e
            yield ("copy", begin, end, m.rng.uniform(100, 1500))
            yield ("write", ev_pulled[r][p], e)

    for r in range(world):
        m.spawn(main(r), f"main{r}")
        m.spawn(comm(r), f"comm{r}")
        for p in peers(r):
            m.spawn(pull(r, p), f"pull{r}<-{p}")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_peer_exchange_protocol_random_schedules(world):
    for seed in range(60):
        rng = random.Random(seed)
        m = Model(seed)
        peer_exchange(m, world, epochs=rng.randint(1, 6))
        m.run()


def test_peer_exchange_model_catches_a_missing_wait():
    """Without the stage's wait for the peers' done flags a rank may rewrite its staging buffer under a pull."""
    with pytest.raises(AssertionError):
        for seed in range(200):
            m = Model(seed)
            peer_exchange(m, 4, epochs=6, skip_done_wait=True)
            m.run()
