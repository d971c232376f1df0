"""Bytes each pointer argument of a C-ABI call must reach, from the argument
meanings in include/tsds.h (shared by the CPU tests that record calls
instead of making them)."""


class TRef:
    """Stands in for a pointer: the tensor (view) it points into."""

    def __init__(self, t):
        self.t = t

    def bytes_left(self):
        st = self.t.untyped_storage()
        return st.nbytes() - (self.t.data_ptr() - st.data_ptr())


def extents(name, a):
    """[(arg index, bytes needed or None if the pointer is unused)] for one call."""
    if name == "tsds_embed":
        ids, stride, table, out, M, N, vocab = a
        return [(0, ((M - 1) * stride + 1) * 8), (2, vocab * N * 2), (3, M * N * 2)]
    if name == "tsds_rms_norm":
        x, w, out, rows, n, ldx, ldo, eps = a
        return [(0, ((rows - 1) * ldx + n) * 2), (1, n * 2), (2, ((rows - 1) * ldo + n) * 2)]
    if name == "tsds_prep_chain":
        base, off, B, T, starts, pos = a
        return [(0, B * 4), (4, B * 4), (5, B * T * 4)]
    if name == "tsds_qk_norm_rope_kv":
        qkv, qn, kn, cos, sin, pos, starts, q, kc, vc, B, T, Hq, Hkv, D, S, rope_len, eps = a
        return [(0, B * T * (Hq + 2 * Hkv) * D * 2), (1, D * 2), (2, D * 2), (3, rope_len * D // 2 * 2),
                (4, rope_len * D // 2 * 2), (5, B * T * 4), (6, B * 4), (7, B * T * Hq * D * 2),
                (8, B * Hkv * S * D * 2), (9, B * Hkv * S * D * 2)]
    if name in ("tsds_linear", "tsds_linear_swiglu", "tsds_linear_f32"):
        x, ldx, W, out, ldo, M, n_out, K, ws, wsb = a
        rows_w = 2 * n_out if name == "tsds_linear_swiglu" else n_out
        eb = 4 if name == "tsds_linear_f32" else 2
        return [(0, ((M - 1) * ldx + K) * 2), (2, rows_w * K * 2), (3, ((M - 1) * ldo + n_out) * eb), (8, wsb)]
    if name in ("tsds_linear_residual", "tsds_linear_bias"):
        x, ldx, W, res, out, ldo, M, n_out, K, ws, wsb = a
        res_b = n_out * 2 if name == "tsds_linear_bias" else ((M - 1) * ldo + n_out) * 2
        return [(0, ((M - 1) * ldx + K) * 2), (2, n_out * K * 2), (3, res_b), (4, ((M - 1) * ldo + n_out) * 2),
                (9, wsb)]
    if name == "tsds_linear_residual_norm":
        x, ldx, W, res, out, ldo, M, n_out, K, nw, nout, nld, eps, ws, wsb = a
        return [(0, ((M - 1) * ldx + K) * 2), (2, n_out * K * 2), (3, ((M - 1) * ldo + n_out) * 2),
                (4, ((M - 1) * ldo + n_out) * 2), (9, n_out * 2), (10, ((M - 1) * nld + n_out) * 2), (13, wsb)]
    if name == "tsds_logits_topk":
        lg, ld, M, V, k, vals, idx, lse = a
        return [(0, ((M - 1) * ld + V) * 2), (5, M * k * 4), (6, M * k * 4), (7, M * 4)]
    if name == "tsds_tree_init":
        states, cur, lengths, tok, frow, pos, mask, starts, B = a
        return [(1, B * 8), (2, B * 4), (3, B * 8), (4, B * 4), (5, B * 4), (6, B * 4), (7, B * 4)]
    if name == "tsds_tree_step":
        states, vals, idx, lse, row_base, T, k, next_T, lengths, tok, frow, pos, mask, starts, B = a
        rows = row_base + B * T
        nt = max(next_T, 1)
        return [(1, rows * k * 4), (2, rows * k * 4), (3, rows * 4), (8, B * 4), (9, B * nt * 8), (10, B * nt * 4),
                (11, B * nt * 4), (12, B * nt * 4), (13, B * 4)]
    if name == "tsds_tree_finalize":
        states, n_nodes, k, lengths, ids, pos, masks, hrow, children, starts, B = a
        NN = n_nodes + 1
        return [(3, B * 4), (4, B * NN * 8), (5, B * NN * 4), (6, B * NN * 4), (7, B * NN * 4),
                (8, B * NN * k * 4), (9, B * 4)]
    if name == "tsds_accept_tree":
        tl, ta, hl, ids, hrow, ch, U, scratch, path, acc, tokens, cur, B, n_nodes, V, k, depth = a
        NN = n_nodes + 1
        return [(0, B * NN * V * 2), (1, B * NN * 8), (2, V * 2), (3, B * NN * 8), (4, B * NN * 4),
                (5, B * NN * k * 4), (6, B * (depth + 1) * (k + 1) * 4), (8, B * (depth + 1) * 4), (9, B * 4),
                (10, B * (depth + 2) * 8), (11, B * 8)]
    if name == "tsds_accept_tree_rule":
        tl, ta, hl, ids, hrow, ch, U, rule, path, acc, tokens, cur, B, n_nodes, V, k, depth = a
        assert rule in (0, 1)
        NN = n_nodes + 1
        return [(0, B * NN * V * 2), (1, B * NN * 8), (2, V * 2), (3, B * NN * 8), (4, B * NN * 4),
                (5, B * NN * k * 4), (6, B * (depth + 1) * (k + 1) * 4), (8, B * (depth + 1) * 4), (9, B * 4),
                (10, B * (depth + 2) * 8), (11, B * 8)]
    if name == "tsds_tree_commit":
        kc, vc, layers, B, Hkv, S, D, lengths, path, acc, depth, hidden, n_nodes, N, root = a
        return [(0, layers * B * Hkv * S * D * 2), (1, layers * B * Hkv * S * D * 2), (7, B * 4),
                (8, B * (depth + 1) * 4), (9, B * 4), (11, B * (n_nodes + 1) * N * 2), (14, B * N * 2)]
    if name == "tsds_eagle_inputs":
        root, hfeat, frow, tok, emb, out, B, T, N, vocab = a
        return [(0, B * N * 2), (2, B * T * 4), (3, B * T * 8), (4, vocab * N * 2), (5, B * T * 2 * N * 2)]
    if name == "tsds_verify_attention":
        q, k, v, out, starts, mask, origin, B, T, Hq, Hkv, D, S, max_kv, split, scale, ws, wsb, status = a
        assert max_kv <= S
        return [(0, B * T * Hq * D * 2), (1, B * Hkv * S * D * 2), (2, B * Hkv * S * D * 2), (3, B * T * Hq * D * 2),
                (4, B * 4), (5, B * T * 4), (16, wsb), (18, 4)]
    if name == "tsds_lm_head_argmax":
        x, ldx, W, logits, am, stride, av, M, V, K, ws, wsb = a
        return [(0, ((M - 1) * ldx + K) * 2), (2, V * K * 2), (3, M * V * 2), (4, ((M - 1) * stride + 1) * 8),
                (6, M * 4), (10, wsb)]
    if name == "tsds_peer_lm_gather":
        bufs, rank, tp, max_elems, xb, rows, vl, val_off, log_off, out, stride, logits, status = a
        assert 0 <= rank < tp and val_off >= 8 * rows
        assert (log_off + 2 * rows * vl if logits is not None else val_off + 4 * rows) <= xb
        return [(9, ((rows - 1) * stride + 1) * 8), (11, rows * tp * vl * 2), (12, 4)]
    if name == "tsds_peer_allreduce_residual":
        x, bufs, rank, tp, slot, M, N, max_elems, status = a
        assert 0 <= rank < tp and slot in (0, 1) and M * N <= max_elems
        return [(0, M * N * 2), (8, 4)]
    if name == "tsds_residual_add_f32":
        x, part, M, N = a
        return [(0, M * N * 2), (1, M * N * 4)]
    if name == "tsds_argmax_merge":
        vals, idx, M, tp, shard, out, stride = a
        return [(0, tp * M * 4), (1, tp * M * 8), (5, ((M - 1) * stride + 1) * 8)]
    if name == "tsds_gather_shards":
        src, dst, tp, M, vs = a
        return [(0, tp * M * vs * 2), (1, M * tp * vs * 2)]
    if name == "tsds_accept_greedy":
        draft, target, acc, tokens, tlen, last, cur, B, K = a
        return [(0, B * K * 8), (1, B * (K + 1) * 8), (2, B * 4), (3, B * (K + 1) * 8), (4, B * 4), (5, B * 8),
                (6, B * 8)]
    if name == "tsds_gather_ids":
        cur, last, draft, vids, d2, B, K = a
        return [(0, B * 8), (1, B * 8), (2, B * K * 8), (3, B * (K + 1) * 8), (4, B * 2 * 8)]
    raise AssertionError(f"no extent rule for {name}")


def fused_extents(a):
    """tsds_fused_layer with its phases / rope given as dicts (see _fused_args):
    [(ref, bytes)] pairs instead of argument indices."""
    phases, n, M, rope, peers, ws, wsb = a
    out = [(ws, wsb)]
    for ph in phases[:n]:
        if ph["kind"] == 2:   # PEER: the residual updated in place (the slots are the peer group's)
            assert peers is not None and ph["n_out"] in (0, 1) and M * ph["K"] <= peers.max_elems
            out.append((ph["out"], ((M - 1) * ph["ldo"] + ph["K"]) * 2))
            continue
        if ph["kind"] == 1:   # NORM
            K = ph["K"]
            out += [(ph["x"], ((M - 1) * ph["ldx"] + K) * 2), (ph["w"], K * 2), (ph["out"], ((M - 1) * ph["ldo"] + K) * 2)]
            continue
        epi, K, n_out = ph["epi"], ph["K"], ph["n_out"]
        rows_w = 2 * n_out if epi == 2 else n_out
        out += [(ph["x"], ((M - 1) * ph["ldx"] + K) * 2), (ph["w"], rows_w * K * 2)]
        if epi != 5:
            out.append((ph["out"], ((M - 1) * ph["ldo"] + n_out) * (4 if epi == 4 else 2)))
        if epi == 1:
            out.append((ph["res"], ((M - 1) * ph["res_ld"] + n_out) * 2))
        if epi == 5:
            r = rope
            assert n_out == (r["Hq"] + 2 * r["Hkv"]) * 128 and M % r["T"] == 0
            B = M // r["T"]
            out += [(r["q_norm_w"], 256), (r["k_norm_w"], 256), (r["cos"], r["rope_len"] * 128),
                    (r["sin"], r["rope_len"] * 128), (r["positions"], M * 4), (r["starts"], B * 4),
                    (r["q_out"], M * r["Hq"] * 256), (r["k_cache"], B * r["Hkv"] * r["S"] * 256),
                    (r["v_cache"], B * r["Hkv"] * r["S"] * 256)]
    return out


def check_call(name, args):
    """Assert every pointer of one recorded call reaches its extent; returns
    the number of pointers checked."""
    n = 0
    pairs = fused_extents(args) if name == "tsds_fused_layer" else [(args[i], need) for i, need in extents(name, args)]
    for ref, need in pairs:
        if ref is None:
            continue
        assert isinstance(ref, TRef), (name, n, ref)
        assert need <= ref.bytes_left(), (name, n, need, ref.bytes_left())
        n += 1
    return n
