"""Measure BASELINE configs 1-4 on one GPU (config 5 is bench.py's line).

    python measure_configs.py [--model-dir DIR] [--out FILE.md]

* config 1  one 512-token Q8_0 sequence: latency (median of 10 after 3 warm-ups), device-resident
            ids (glp_embed_packed_device) and host ids -> host embeddings (glp_embed_tokens);
* config 2  Q8_0 x bf16 GEMM (glp_q8_0_gemm: dequantisation of the Q8_0 weight into the library's
            scratch + the tcgen05 GEMM), W [N,K] in {768x768, 256x768, 1152x768, 768x1152},
            M in {512, 4096, 32768, 131072}, bf16 out; % of roofline = max(FLOP / P_tensor,
            bytes / BW_HBM) / time with the measured peaks of MEASURED_PEAKS.json (burst);
* config 3  256 Q8_0 sequences, lengths uniform in [64, 512], 768-d and 256-d MRL outputs:
            embeddings/s and TFLOP/s of valid-token work (padding is not computed);
* serving   the dynamic-batching engine (glp_engine_*): client threads each embedding single
            512-token Q8_0 sequences through InferenceEngine; requests/s, batch sizes and
            per-request latency percentiles (host wall clock: end to end);
* text      texts -> embeddings (glp_embed_texts): the host tokenizer's throughput on 1 and all
            cores (and the `tokenizers` library's per-text loop, the reference's sequential
            tokenisation, when importable), then 256 synthetic ~512-token texts end to end with the
            BPE vocabulary of tests/golden/tokenizer_golden.json written into the model file;
* config 4  BF16 weights, one 8192-token sequence (sliding window 512 on local layers, full on
            global): latency, then per-kernel ms / TFLOP/s / GB/s from the library's own CUDA-event
            profile (a separate pass, so the latency carries no profiling overhead);
* ple       an EmbeddingGemma-2-shaped Q8_0 model (hidden 512, FFN 2048, 4 query heads over 2 KV
            heads on sliding layers and 1 on global ones, per-layer embeddings of 512, head 512 ->
            768; head_dim 256 on every layer): 1,024 sequences of 512 tokens, embeddings/s and the
            per-kernel profile.

All inputs are the seeded synthetic GGUFs of glypr_b200.synth; times are CUDA events on the
launching stream.  Prints a markdown report (and writes it with --out).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from glypr_b200 import api, synth  # noqa: E402
from bench import ClockSampler  # noqa: E402

GFLOP_PER_SEQ_512 = 123.21  # linear + attention + head per 512-token sequence (config 1)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json, burst)"
    return 1590.0, 6650.0, "fallback"


def timed(torch, fn, warm=3, reps=10):
    """Median ms of `fn` over `reps` runs after `warm` warm-ups (CUDA events, current stream)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return float(np.median(ts))


def linear_flops_per_token(cfg) -> float:
    d, h, f = cfg.head_dim, cfg.hidden, cfg.ffn
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * d
    per_layer = qkv * h + h * cfg.n_heads * d + 2 * f * h + h * f
    return 2.0 * per_layer * cfg.n_layers


def attention_flops(cfg, lengths, window=512) -> float:
    """4 * head_dim * heads FLOP per visible (query, key) pair, sliding layers windowed."""
    total = 0.0
    for L in lengths:
        full = float(L) * L
        if window > 0 and L > window + 1:
            i = np.arange(L)
            vis = (np.minimum(L - 1, i + window) - np.maximum(0, i - window) + 1).sum()
        else:
            vis = full
        n_global = sum(1 for li in range(cfg.n_layers) if not cfg.layer_is_sliding(li))
        total += (cfg.n_layers - n_global) * vis + n_global * full
    return 4.0 * cfg.head_dim * cfg.n_heads * total


def packed_inputs(torch, ids, lengths):
    valid = np.concatenate([ids[i, : lengths[i]] for i in range(len(lengths))]).astype(np.int32)
    h_cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return torch.from_numpy(valid).cuda(), torch.from_numpy(h_cu).cuda(), h_cu


def config1(torch, emb, report):
    ids, lens = synth.make_batch(1, 512, emb.info.vocab, seed=synth.MASTER_SEED + 11)
    d_ids, d_cu, h_cu = packed_inputs(torch, ids, lens)
    d_out = torch.empty((1, 768), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    dev_ms = timed(torch, lambda: emb.embed_packed_device(d_ids.data_ptr(), d_cu.data_ptr(), h_cu, 1, 768,
                                                         d_out.data_ptr(), stream))
    host_ms = timed(torch, lambda: emb.embed_tokens(ids, lens))
    report.append("## Config 1 — one 512-token Q8_0 sequence\n")
    report.append("| path | latency (ms, median of 10) | TFLOP/s |\n|---|---:|---:|")
    for name, ms in (("device-resident ids (`glp_embed_packed_device`)", dev_ms),
                     ("host ids → host embedding (`glp_embed_tokens`)", host_ms)):
        report.append(f"| {name} | {ms:.3f} | {GFLOP_PER_SEQ_512 / ms:.1f} |")
    report.append("")


def config2(torch, report):
    """glp_q8_0_gemm: the default route and both forced routes (GLP_Q8_GEMM, read per call)."""
    p_t, p_b, src = peaks()
    report.append("## Config 2 — Q8_0 × bf16 GEMM (`glp_q8_0_gemm`, bf16 out)\n")
    report.append(f"Peaks: {p_t:.0f} TFLOP/s, {p_b:.0f} GB/s ({src}). Times are per call (CUDA events, "
                  "median of 10 after 3 warm-ups). Routes: *fused* = one launch streaming the raw Q8_0 rows "
                  "by TMA and dequantising in shared memory; *two-pass* = dequantise into library scratch, "
                  "then the bf16 CTA-pair GEMM; *default* = fused up to M = 8,192, two-pass above.\n")
    report.append("| W [N×K] | M | default ms | % of roofline | fused ms | two-pass ms |\n"
                  "|---|---:|---:|---:|---:|---:|")
    rng = np.random.default_rng(synth.MASTER_SEED + 22)
    st = torch.cuda.current_stream().cuda_stream  # the stream the timing events are recorded on
    for n, k in ((768, 768), (256, 768), (1152, 768), (768, 1152)):
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        blocks = synth.quantize_q8_0(w)
        d_w = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
        for m in (512, 4096, 32768, 131072):
            x = torch.randn((m, k), device="cuda").to(torch.bfloat16)
            y = torch.empty((m, n), device="cuda", dtype=torch.bfloat16)
            ms = {}
            for route in ("default", "fused", "two-pass"):
                if route == "default":
                    os.environ.pop("GLP_Q8_GEMM", None)
                else:
                    os.environ["GLP_Q8_GEMM"] = route
                ms[route] = timed(torch, lambda: api.q8_0_gemm(d_w.data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(),
                                                                 False, st))
            os.environ.pop("GLP_Q8_GEMM", None)
            flop = 2.0 * m * n * k
            byts = n * k / 32 * 34 + 2.0 * m * k + 2.0 * m * n
            roof_ms = max(flop / (p_t * 1e9), byts / (p_b * 1e6))
            report.append(f"| {n}×{k} | {m} | {ms['default']:.4f} | {100 * roof_ms / ms['default']:.1f} | "
                          f"{ms['fused']:.4f} | {ms['two-pass']:.4f} |")
            del x, y
    report.append("")


def attention_ab(torch, report):
    """glp_flash_attention on the bench's shapes: the CTA-pair kernel (default) against the
    one-CTA kernel (GLP_ATTENTION=single), same inputs."""
    p_t, _, src = peaks()
    report.append("## Attention — CTA-pair kernel vs one-CTA kernel (`glp_flash_attention`, head_dim 256)\n")
    report.append(f"3 query heads over 1 KV head, f16 qkv with unit-RMS q/k scaled to logit std 16 (the BASELINE "
                  f"init's spread); median of 10 calls; TFLOP/s of the visible (query, key) pairs, peak {p_t:.0f} ({src}).\n")
    report.append("| sequences x length | window | pair ms | pair TFLOP/s | single ms | single TFLOP/s |\n"
                  "|---|---:|---:|---:|---:|---:|")
    rng = np.random.default_rng(synth.MASTER_SEED + 66)
    for n_seq, L in ((512, 512), (1, 8192)):
        t = n_seq * L
        qkv = rng.standard_normal((t, 5 * 256), dtype=np.float32)
        d_qkv = torch.from_numpy(qkv.astype(np.float16)).cuda()
        d_cu = torch.from_numpy(np.arange(0, (n_seq + 1) * L, L, dtype=np.int32)).cuda()
        out = torch.empty((t, 3 * 256), dtype=torch.float16, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        for window in (0, 512):
            if window:
                i = np.arange(L)
                vis = float((np.minimum(L - 1, i + window) - np.maximum(0, i - window) + 1).sum()) * n_seq
            else:
                vis = float(L) * L * n_seq
            flop = 4.0 * 256 * 3 * vis
            ms = {}
            for route in ("pair", "single"):
                if route == "single":
                    os.environ["GLP_ATTENTION"] = "single"
                else:
                    os.environ.pop("GLP_ATTENTION", None)
                ms[route] = timed(torch, lambda: api.flash_attention(d_qkv.data_ptr(), d_cu.data_ptr(), n_seq, L, 3, 1,
                                                                     256, window, out.data_ptr(), st))
            os.environ.pop("GLP_ATTENTION", None)
            report.append(f"| {n_seq} x {L} | {window} | {ms['pair']:.3f} | {flop / ms['pair'] / 1e9:.0f} | "
                          f"{ms['single']:.3f} | {flop / ms['single'] / 1e9:.0f} |")
        del d_qkv, out
    report.append("")


def q8_one(torch, spec):
    """One glp_q8_0_gemm shape on one route, 5 calls (a small case for ncu): N,K,M,route."""
    n, k, m, route = spec.split(",")
    n, k, m = int(n), int(k), int(m)
    os.environ["GLP_Q8_GEMM"] = route
    rng = np.random.default_rng(synth.MASTER_SEED + 22)
    blocks = synth.quantize_q8_0(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    d_w = torch.from_numpy(blocks.view(np.uint8).reshape(-1).copy()).cuda()
    x = torch.randn((m, k), device="cuda").to(torch.bfloat16)
    y = torch.empty((m, n), device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    ms = timed(torch, lambda: api.q8_0_gemm(d_w.data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(), False, st),
               warm=2, reps=3)
    print(f"{n}x{k} M={m} {route}: {ms * 1e3:.1f} us, {2.0 * m * n * k / ms / 1e9:.0f} TFLOP/s, "
          f"status {api.kernel_status(0)}")


def config3(torch, emb, report):
    rng = np.random.default_rng(synth.MASTER_SEED + 33)
    lens = rng.integers(64, 513, size=256).astype(np.int32)
    ids, lens = synth.make_batch(256, 512, emb.info.vocab, seed=synth.MASTER_SEED + 34, lengths=list(lens))
    d_ids, d_cu, h_cu = packed_inputs(torch, ids, lens)
    stream = torch.cuda.current_stream().cuda_stream
    d768 = torch.empty((256, 768), dtype=torch.float32, device="cuda")
    d256 = torch.empty((256, 256), dtype=torch.float32, device="cuda")
    ms768 = timed(torch, lambda: emb.embed_packed_device(d_ids.data_ptr(), d_cu.data_ptr(), h_cu, 256, 768,
                                                        d768.data_ptr(), stream))
    ms256 = timed(torch, lambda: emb.embed_packed_device(d_ids.data_ptr(), d_cu.data_ptr(), h_cu, 256, 256,
                                                        d256.data_ptr(), stream))
    host_ms = timed(torch, lambda: emb.embed_tokens(ids, lens))
    cfg = synth.BASELINE
    tok = float(lens.sum())
    flop = linear_flops_per_token(cfg) * tok + attention_flops(cfg, lens)
    report.append("## Config 3 — 256 Q8_0 sequences, lengths uniform in [64, 512]\n")
    report.append(f"Valid tokens {int(tok)} (mean length {tok / 256:.1f}); valid-token work "
                  f"{flop / 1e12:.2f} TFLOP per batch (padding is never computed: packed by length).\n")
    report.append("| output | ms per batch | embeddings/s | tokens/s | TFLOP/s |\n|---|---:|---:|---:|---:|")
    for name, ms in (("768-d (device-resident ids)", ms768), ("256-d MRL (device-resident ids)", ms256),
                     ("768-d, host ids → host embeddings", host_ms)):
        report.append(f"| {name} | {ms:.2f} | {256 / ms * 1e3:.0f} | {tok / ms * 1e3 / 1e6:.2f} M | "
                      f"{flop / ms / 1e9:.0f} |")
    report.append("")


def config4(torch, path, report):
    with api.GlyprEmbedder.load_gguf(path, [0]) as emb:
        ids, lens = synth.make_batch(1, 8192, emb.info.vocab, seed=synth.MASTER_SEED + 44)
        d_ids, d_cu, h_cu = packed_inputs(torch, ids, lens)
        d_out = torch.empty((1, 768), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        run = lambda: emb.embed_packed_device(d_ids.data_ptr(), d_cu.data_ptr(), h_cu, 1, 768, d_out.data_ptr(),
                                              stream)
        ms = timed(torch, run)
        host_ms = timed(torch, lambda: emb.embed_tokens(ids, lens), warm=2, reps=5)
        emb.profile_enable(True)
        run()
        torch.cuda.synchronize()
        prof = emb.profile_read()
        emb.profile_enable(False)
    cfg = synth.BASELINE
    flop = linear_flops_per_token(cfg) * 8192 + attention_flops(cfg, [8192])
    report.append("## Config 4 — BF16 weights, one 8192-token sequence\n")
    report.append(f"Work {flop / 1e12:.3f} TFLOP (linear + windowed local / full global attention). "
                  f"Latency {ms:.2f} ms device-resident ({flop / ms / 1e9:.0f} TFLOP/s), {host_ms:.2f} ms "
                  "with host ids in and the host embedding out.\n")
    report.append("Per kernel (one forward, library CUDA-event profile):\n")
    report.append("| kernel | launches | ms | TFLOP/s | GB/s |\n|---|---:|---:|---:|---:|")
    for name, v in sorted(((k, v) for k, v in prof.items() if not k.startswith("_")), key=lambda kv: -kv[1]["ms"]):
        if v["launches"] == 0:
            continue
        tf = f"{v['flops'] / v['ms'] / 1e9:.0f}" if v["flops"] > 0 else "—"
        gb = f"{v['bytes'] / v['ms'] / 1e6:.0f}" if v["bytes"] > 0 else "—"
        report.append(f"| {name} | {v['launches']} | {v['ms']:.3f} | {tf} | {gb} |")
    report.append("")


EMBEDDINGGEMMA2_SHAPE = synth.EncoderConfig(hidden=512, ffn=2048, n_heads=4, n_kv_heads=2, global_kv_heads=1,
                                            head_dims=(768,), ple_dim=512, global_head_dim=512)


def ple_config(torch, path, report, n=1024):
    with api.GlyprEmbedder.load_gguf(path, [0]) as emb:
        ids, lens = synth.make_batch(n, 512, emb.info.vocab, seed=synth.MASTER_SEED + 55)
        d_ids, d_cu, h_cu = packed_inputs(torch, ids, lens)
        d_out = torch.empty((n, 768), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        run = lambda: emb.embed_packed_device(d_ids.data_ptr(), d_cu.data_ptr(), h_cu, n, 768, d_out.data_ptr(),
                                              stream)
        ms = timed(torch, run, warm=3, reps=5)
        emb.profile_enable(True)
        run()
        torch.cuda.synchronize()
        prof = emb.profile_read()
        emb.profile_enable(False)
    total = sum(v["ms"] for k, v in prof.items() if not k.startswith("_"))
    report.append("## Per-layer embeddings — EmbeddingGemma-2-shaped Q8_0 model, 512-token sequences\n")
    report.append(f"24 layers, hidden 512, FFN 2048, 4 query heads over 2 KV heads of 256 on the sliding layers "
                  f"and 1 KV head of 512 on the global layers (EmbeddingGemma 2's widths), per-layer inputs of "
                  f"512, head 512 -> 768. {n} sequences: "
                  f"{ms:.1f} ms per batch, {n / ms * 1e3:.0f} embeddings/s (device-resident ids).\n")
    report.append("Per kernel (one batch, library CUDA-event profile):\n")
    report.append("| kernel | launches | ms | share | TFLOP/s | GB/s |\n|---|---:|---:|---:|---:|---:|")
    for name, v in sorted(((k, v) for k, v in prof.items() if not k.startswith("_")), key=lambda kv: -kv[1]["ms"]):
        if v["launches"] == 0:
            continue
        tf = f"{v['flops'] / v['ms'] / 1e9:.0f}" if v["flops"] > 0 else "—"
        gb = f"{v['bytes'] / v['ms'] / 1e6:.0f}" if v["bytes"] > 0 else "—"
        report.append(f"| {name} | {v['launches']} | {v['ms']:.3f} | {v['ms'] / total:.3f} | {tf} | {gb} |")
    report.append("")


def serving(emb, report, clients=64, per_client=64, max_batch=512):
    import threading
    ids, lens = synth.make_batch(clients * per_client, 512, emb.info.vocab, seed=synth.MASTER_SEED + 55)
    lat = []
    lock = threading.Lock()
    with api.InferenceEngine(emb, max_batch_size=max_batch) as eng:
        eng.embed(ids[0])  # warm-up (graph capture of the first shapes)

        def client(c):
            mine = []
            for k in range(per_client):
                i = c * per_client + k
                t0 = time.perf_counter()
                eng.embed(ids[i])
                mine.append(time.perf_counter() - t0)
            with lock:
                lat.extend(mine)

        threads = [threading.Thread(target=client, args=(c,)) for c in range(clients)]
        t0 = time.perf_counter()
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        wall = time.perf_counter() - t0
        st = eng.stats()
    n = clients * per_client
    lat_ms = np.sort(np.array(lat)) * 1e3
    report.append("## Serving — dynamic-batching engine, single 512-token requests\n")
    report.append(f"{clients} client threads x {per_client} requests, max_batch {max_batch} "
                  f"(glp_engine_embed: the reference server's batching policy, engine.rs:216-245).\n")
    report.append("| requests/s | batches | mean batch | largest batch | latency p50 (ms) | p99 (ms) |\n"
                  "|---:|---:|---:|---:|---:|---:|")
    report.append(f"| {n / wall:.0f} | {st['batches'] - 1} | {(st['requests'] - 1) / max(st['batches'] - 1, 1):.1f} | "
                  f"{st['largest_batch']} | {lat_ms[len(lat_ms) // 2]:.1f} | {lat_ms[int(len(lat_ms) * 0.99)]:.1f} |")
    report.append("")


def _synthetic_texts(n, n_words, seed):
    rng = np.random.default_rng(seed)
    syl = ["ka", "lo", "mi", "ne", "ru", "sta", "tion", "er", "ing", "the", "and", "qu", "str", "ph", "ed",
           "é", "ü", "ß", "κα", "σο", "при", "вет", "東京", "研究", "3.14", "(a,b)", "->", "🙂"]
    out = []
    for _ in range(n):
        words = ["".join(rng.choice(syl, size=rng.integers(1, 4))) for _ in range(n_words)]
        out.append(" ".join(words))
    return out


def text_path(torch, model_dir, report, n_texts=256):
    golden = os.path.join(ROOT, "tests", "golden", "tokenizer_golden.json")
    vocab = next(s for s in json.load(open(golden, encoding="utf-8"))["sets"] if s["name"] == "trained")
    path = os.path.join(model_dir, "baseline_q8_0_bpe.gguf")
    if not os.path.exists(path):
        synth.write_gguf(path, synth.BASELINE, tokenizer=(vocab["tokens"], vocab["merges"]))
    texts = _synthetic_texts(n_texts, 220, synth.MASTER_SEED + 77)
    nbytes = sum(len(t.encode()) for t in texts)

    def best(fn, reps=5):
        t = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            t.append(time.perf_counter() - t0)
        return min(t)

    with api.Tokenizer.from_gguf(path) as tok:
        ids = tok.encode_batch(texts, api.GLP_TOKENS_SEQUENCE)
        n_ids = sum(len(r) for r in ids)
        rows = [("glp_tokenize_batch, 1 thread", best(lambda: tok.encode_batch(texts, 2, n_threads=1)))]
        rows.append((f"glp_tokenize_batch, all {os.cpu_count()} host threads",
                     best(lambda: tok.encode_batch(texts, 2, n_threads=0))))
        try:
            from tokenizers import Tokenizer, models, normalizers, pre_tokenizers
            v = {}
            for i, t in enumerate(vocab["tokens"]):
                v[t] = i
            lib = Tokenizer(models.BPE(vocab=v, merges=[tuple(m.split(" ")) for m in vocab["merges"]],
                                       unk_token="<unk>", fuse_unk=True, byte_fallback=True))
            lib.normalizer = normalizers.Replace(" ", "\u2581")
            lib.pre_tokenizer = pre_tokenizers.Split(" ", behavior="merged_with_previous", invert=False)
            rows.append(("`tokenizers` 0.22 per-text loop (the reference's tokenisation), 1 thread",
                         best(lambda: [lib.encode(t) for t in texts], 3)))
        except ImportError:
            pass
        report.append("## Text front end — host tokenizer and texts -> embeddings\n")
        report.append(f"{n_texts} synthetic texts, {nbytes / n_texts:.0f} bytes and {n_ids / n_texts:.0f} ids each "
                      f"(BPE vocabulary of {len(vocab['tokens'])} tokens, {len(vocab['merges'])} merges).\n")
        report.append("| tokenizer | ms per batch | MB/s | ids/s |\n|---|---:|---:|---:|")
        for name, t in rows:
            report.append(f"| {name} | {t * 1e3:.1f} | {nbytes / t / 1e6:.1f} | {n_ids / t / 1e6:.2f} M |")
        report.append("")
        report.append("| texts | tokenise (all host threads), ms | glp_embed_tokens on the ids, ms | "
                      "glp_embed_texts, ms | embeddings/s | tokenisation hidden, ms |\n|---:|---:|---:|---:|---:|---:|")
        with api.GlyprEmbedder.load_gguf(path, [0]) as emb:
            for n in (n_texts, 8 * n_texts):
                batch = (texts * 8)[:n]
                rows_n = tok.encode_batch(batch, api.GLP_TOKENS_SEQUENCE)
                lens = np.array([len(r) for r in rows_n], np.int32)
                padded = np.zeros((n, int(lens.max())), np.int32)
                for i, r in enumerate(rows_n):
                    padded[i, :len(r)] = r
                for _ in range(2):
                    emb.embed_texts(tok, batch)
                reps = 5 if n <= n_texts else 3
                t_tok = best(lambda: tok.encode_batch(batch, api.GLP_TOKENS_SEQUENCE, n_threads=0), reps)
                t_all = best(lambda: emb.embed_texts(tok, batch), reps)
                t_ids = best(lambda: emb.embed_tokens(padded, lens), reps)
                # glp_embed_texts tokenises the next part of a large batch while the current part
                # embeds: the time it saves against tokenising everything first
                report.append(f"| {n} | {t_tok * 1e3:.1f} | {t_ids * 1e3:.1f} | {t_all * 1e3:.1f} | "
                              f"{n / t_all:.0f} | {(t_tok + t_ids - t_all) * 1e3:.1f} |")
        report.append("")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model-dir", default=os.environ.get("GLYPR_BENCH_DIR", "/tmp/glypr_models"))
    ap.add_argument("--out", default=None)
    ap.add_argument("--configs", default="1,2,3,4,serving")
    ap.add_argument("--q8-one", default=None, help="N,K,M,route: one glp_q8_0_gemm case (for ncu), nothing else")
    args = ap.parse_args(argv)
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    if args.q8_one:
        api.load_library()
        q8_one(torch, args.q8_one)
        return
    os.makedirs(args.model_dir, exist_ok=True)
    want = set(int(c) if c.isdigit() else c for c in args.configs.split(","))
    report = [f"# BASELINE configs 1–4 on one {torch.cuda.get_device_name(0)}\n",
              f"Command: `python measure_configs.py --configs {args.configs}` "
              f"({time.strftime('%Y-%m-%d')}); median of 10 runs after 3 warm-ups unless stated.\n"]
    api.load_library()
    # a stream of our own: the library runs repeated launch-chunk shapes as CUDA graphs, which
    # the legacy default stream cannot hold
    side = torch.cuda.Stream()
    torch.cuda.set_stream(side)
    clocks = ClockSampler(0)
    clocks.start()
    if want & {1, 3, "serving"}:
        q8 = synth.ensure_gguf(os.path.join(args.model_dir, "baseline_q8_0.gguf"), synth.BASELINE)
        with api.GlyprEmbedder.load_gguf(q8, [0]) as emb:
            if 1 in want:
                config1(torch, emb, report)
            if 3 in want:
                config3(torch, emb, report)
            if "serving" in want:
                serving(emb, report)
    if "text" in want:
        text_path(torch, args.model_dir, report)
    if 2 in want:
        config2(torch, report)
    if "attn" in want:
        attention_ab(torch, report)
    if "ple" in want:
        pl = synth.ensure_gguf(os.path.join(args.model_dir, "embeddinggemma2_shape_q8_0.gguf"), EMBEDDINGGEMMA2_SHAPE)
        ple_config(torch, pl, report)
    if 4 in want:
        bf = synth.ensure_gguf(os.path.join(args.model_dir, "baseline_bf16.gguf"),
                               synth.EncoderConfig(weight_type="bf16"))
        config4(torch, bf, report)
    clk = clocks.stop()
    report.append(f"Clocks over the whole run (nvidia-smi every 200 ms, samples under load): median SM "
                  f"{clk.get('sm_mhz')} MHz of {clk.get('sm_max_mhz')} MHz, max power {clk.get('power_w_max')} W, "
                  f"throttle reasons {clk.get('reasons')}.\n")
    text = "\n".join(report)
    print(text, flush=True)
    if args.out:
        with open(args.out, "w") as f:
            f.write(text + "\n")


if __name__ == "__main__":
    main()
