"""Shared test helpers: run the CPU oracle on a workload Batch."""

import numpy as np
import torch

import oracle as O


def np_f32(t):
    return t.detach().float().cpu().numpy()


def np_i(t):
    return t.detach().cpu().numpy()


def oracle_verify(batch, nthreads=None):
    """The oracle's five outputs for a workloads.Batch (any device)."""
    return O.verify_logits(
        np_i(batch.candidates), np_f32(batch.target_logits), np_i(batch.target_rows),
        None if batch.draft_logits is None else np_f32(batch.draft_logits),
        None if batch.draft_rows is None else np_i(batch.draft_rows),
        np_f32(batch.temperature), np_i(batch.top_k), np_f32(batch.top_p),
        np_i(batch.verify_lens), np_f32(batch.uniforms), np_f32(batch.uniform_final),
        np_i(batch.prefix_lens), nthreads=nthreads)


NAMES = ("accept", "commit", "bonus", "output", "new_seq")


def assert_same(got, expected, tag=""):
    for name, g, e in zip(NAMES, got, expected):
        g = g.detach().cpu().numpy() if isinstance(g, torch.Tensor) else np.asarray(g)
        if not np.array_equal(g, e):
            bad = np.argwhere(g != e)[:8]
            raise AssertionError(f"{tag} {name} differs at {bad.tolist()}: got {g[tuple(bad.T)]} "
                                 f"expected {e[tuple(bad.T)]}")


# ---- serial chain fixtures (tests/golden/serial.npz) ----------------------------------------

def serial_chain_case(d, ci):
    """Inputs and reference outputs of sampled-chain case ci."""
    get = lambda name: d[f"c{ci}_{name}"]  # noqa: E731
    inputs = dict(table=get("table"), inv_t=get("inv_t"), top_k=get("top_k"), top_p=get("top_p"),
                  min_p=get("min_p"), greedy=get("greedy"), u=get("u"), cand=get("cand"),
                  greedy_tok=get("gtok"), T=int(get("T")))
    return inputs, dict(tok=get("tok"), q=get("q"), conf=get("conf"), ref_tok=get("ref_tok"),
                        ref_q=get("ref_q"))


def bf16_from_bits(a):
    """float32 values of bf16 bit patterns stored as int16."""
    return (np.asarray(a).astype(np.int32).astype(np.uint32) << 16).view(np.float32)


def serial_table_case(d, ti):
    """Dense inputs of greedy-table case ti: the stored table rows (candidate and sender ids)
    are placed at their ids in zero-filled [V, ...] arrays (no other row is ever read)."""
    get = lambda name: d[f"t{ti}_{name}"]  # noqa: E731
    bs, T, H, R, C, V, k, head = (int(x) for x in get("dims"))
    used = get("used")
    lm = np.zeros((V, H), np.float32)
    tg = np.zeros((V, R), np.float32)
    tsv = np.zeros((V, 2 * R), np.float32)
    lm[used] = bf16_from_bits(get("lm"))
    tg[used] = bf16_from_bits(get("tg"))
    tsv[used] = bf16_from_bits(get("tsv"))
    case = dict(bs=bs, T=T, H=H, R=R, V=V, k=k, head=bool(head),
                raw=bf16_from_bits(get("raw")), norm_w=bf16_from_bits(get("norm_w")),
                gb=bf16_from_bits(get("gb")), query=bf16_from_bits(get("query")),
                rms=get("rms").astype(np.float32), cand=get("cand"), input_ids=get("input_ids"),
                lm=lm, tg=tg, tsv=tsv)
    ref = dict(idx=get("idx"), conf=get("conf"), chain=get("chain"), chain_conf=get("chain_conf"),
               ref_table=get("ref_table"))
    return case, ref


def serial_scores(case):
    """Oracle scores and error scale of a greedy-table case."""
    import oracle.serial as OS

    cand = case["cand"]
    k = case["k"]
    lm = case["lm"]
    return OS.table_scores(case["raw"], case["norm_w"], cand, case["input_ids"],
                           lambda nn: lm[cand[nn]], case["tg"], case["tsv"], case["query"],
                           case["rms"], case["gb"], case["T"])
