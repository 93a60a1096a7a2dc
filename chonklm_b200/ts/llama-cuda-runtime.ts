// Bun FFI host binding of libchonk_b200.so: the llama-webgpu runtime's module
// API (src/lib/llama-wgsl-runtime.ts:174-324) on the B200 engine.
//
// Drop-in for RUNTIMES["llama-webgpu"] (src/components/ModelDashboard.ts:109-116):
//   loadLlamaCudaModel(model, onProgress?, onStep?)   <- loadLlamaWgslModel :184-240
//   generateLlamaCuda(loaded, promptIds, opts)        <- generateLlamaWgsl :242-314
//   disposeLlamaCuda(loaded)                          <- disposeLlamaWgsl :316-318
//   resetLlamaCudaConversation(loaded)                <- resetLlamaWgslConversation :320-324
// The engine surface (runToken / reset / position / dispose) is CudaEngine.
//
// It reuses the reference's own GGUF manifest rules and range loader; the
// reference side exports three internals of llama-wgsl-runtime.ts for it:
// `buildGgufLlamaManifest` (:326-425), `modelFileUrl` (:427-429) and the
// `LlamaManifest` type (:36-72).  Calls are synchronous and throw the
// engine's message on a non-zero status, as the reference throws.  Written
// for Bun (bun:ffi); there is no JavaScript runtime on the machines this
// repository is built and tested on, so this file has not been executed: its
// struct layouts are checked against the C ABI by tests/test_abi_cpu.py.

import { dlopen, FFIType, ptr, CString } from "bun:ffi";
import type { LoadStepCallback, ProgressCallback } from "./cache";
import { fetchCachedRange } from "./cache";
import { buildGgufLlamaManifest, modelFileUrl, type LlamaManifest } from "./llama-wgsl-runtime";
import type { ModelDef } from "./registry";
import { needsSamplingReadback, type SamplingOptions } from "./sampling";
import { Tokenizer } from "./tokenizer";

const lib = dlopen(process.env.CHONK_B200_LIB ?? "libchonk_b200.so", {
  ck_create: { args: [FFIType.ptr, FFIType.i32, FFIType.ptr], returns: FFIType.i32 },
  ck_upload_tensor: {
    args: [FFIType.ptr, FFIType.cstring, FFIType.i32, FFIType.ptr, FFIType.i32, FFIType.ptr, FFIType.u64],
    returns: FFIType.i32,
  },
  ck_finalize: { args: [FFIType.ptr], returns: FFIType.i32 },
  ck_run_token: { args: [FFIType.ptr, FFIType.u32, FFIType.i32, FFIType.ptr, FFIType.ptr], returns: FFIType.i32 },
  ck_prefill: {
    args: [FFIType.ptr, FFIType.ptr, FFIType.i32, FFIType.i32, FFIType.ptr, FFIType.ptr],
    returns: FFIType.i32,
  },
  ck_decode: {
    args: [FFIType.ptr, FFIType.u32, FFIType.i32, FFIType.ptr, FFIType.ptr, FFIType.i32, FFIType.ptr, FFIType.ptr],
    returns: FFIType.i32,
  },
  ck_reset: { args: [FFIType.ptr], returns: FFIType.i32 },
  ck_set_sampler: { args: [FFIType.ptr, FFIType.i32], returns: FFIType.i32 },
  ck_position: { args: [FFIType.ptr, FFIType.ptr], returns: FFIType.i32 },
  ck_destroy: { args: [FFIType.ptr], returns: FFIType.i32 },
  ck_last_error: { args: [FFIType.ptr], returns: FFIType.cstring },
  ck_global_error: { args: [], returns: FFIType.cstring },
  ck_abi_info: { args: [FFIType.ptr, FFIType.ptr], returns: FFIType.void },
});
const S = lib.symbols;

// ---- struct layouts of include/chonk_b200.h (byte offsets) ----------------------
export const CK_MAX_LAYERS = 128;
export const CK_CFG_SIZE = 1084;
export const CK_CFG_LAYOUT = {
  hidden: 0, intermediate: 4, vocab: 8, layers: 12, heads: 16, kv_heads: 20, head_dim: 24, context_length: 28,
  norm_eps: 32, qk_norm_eps: 36, embedding_scale: 40, arch: 44, rope_interleaved: 48, qk_norm: 52, kv_dtype: 56,
  layer_rope_theta: 60, layer_window: 572,
} as const;
export const CK_SAMPLING_SIZE = 64;
export const CK_SAMPLING_LAYOUT = {
  temperature: 0, top_p: 8, top_k: 16, repetition_penalty: 24, penalized_ids: 32, n_penalized: 40,
  philox_seed: 48, philox_offset: 56,
} as const;
const CK_ARCH_LLAMA = 0, CK_ARCH_GEMMA3 = 1, CK_KV_F16 = 0, CK_KV_F32 = 1, CK_ECONTEXT = -4;

const GGML_OF_DTYPE: Record<string, number> = {
  float32: 0, float16: 1, "gguf-q5_0": 6, "gguf-q5_1": 7, "gguf-q8_0": 8, "gguf-q4_k": 12, "gguf-q6_k": 14,
};

(() => {   // the library's own sizes must match this file's layouts
  const a = new Int32Array(2);
  S.ck_abi_info(ptr(a), ptr(a.subarray(1)));
  if (a[0] !== CK_CFG_SIZE || a[1] !== CK_SAMPLING_SIZE) {
    throw new Error(`libchonk_b200 ABI mismatch: cfg ${a[0]} / sampling ${a[1]} bytes`);
  }
})();

function check(h: number | null, rc: number): void {
  if (rc === 0) return;
  const msg = String(h === null ? S.ck_global_error() : S.ck_last_error(h));
  throw new Error(msg || `libchonk_b200 error ${rc}`);
}

function packCfg(m: LlamaManifest["model"], contextLength: number, kvDtype: string | undefined): Uint8Array {
  const buf = new ArrayBuffer(CK_CFG_SIZE);
  const v = new DataView(buf);
  const L = CK_CFG_LAYOUT;
  if (m.layers > CK_MAX_LAYERS) throw new Error(`${m.layers} layers exceeds ${CK_MAX_LAYERS}`);
  v.setInt32(L.hidden, m.hidden, true);
  v.setInt32(L.intermediate, m.intermediate, true);
  v.setInt32(L.vocab, m.vocab, true);
  v.setInt32(L.layers, m.layers, true);
  v.setInt32(L.heads, m.heads, true);
  v.setInt32(L.kv_heads, m.kvHeads, true);
  v.setInt32(L.head_dim, m.headDim, true);
  v.setInt32(L.context_length, contextLength, true);
  v.setFloat32(L.norm_eps, m.normEps, true);
  v.setFloat32(L.qk_norm_eps, m.qkNormEps ?? m.normEps, true);
  v.setFloat32(L.embedding_scale, m.embeddingScale ?? 1, true);
  v.setInt32(L.arch, m.architecture === "gemma3" ? CK_ARCH_GEMMA3 : CK_ARCH_LLAMA, true);
  v.setInt32(L.rope_interleaved, m.ropeLayout === "interleaved" ? 1 : 0, true);
  v.setInt32(L.qk_norm, m.qkNorm ? 1 : 0, true);
  v.setInt32(L.kv_dtype, kvDtype === "float32" ? CK_KV_F32 : CK_KV_F16, true);
  for (let i = 0; i < m.layers; i++) {
    v.setUint32(L.layer_rope_theta + 4 * i, Math.round(m.layerRopeTheta?.[i] ?? m.ropeTheta), true);   // :1477
    v.setUint32(L.layer_window + 4 * i, m.layerAttentionWindow?.[i] ?? 0, true);
  }
  return new Uint8Array(buf);
}

// Keeps the penalty id array alive while the struct points at it.
interface PackedSampling { bytes: Uint8Array; keep: Uint32Array | null }

function packSampling(o: SamplingOptions & { seed?: number; penalizedTokenIds?: number[] },
                      offset: number): PackedSampling {
  const buf = new ArrayBuffer(CK_SAMPLING_SIZE);
  const v = new DataView(buf);
  const L = CK_SAMPLING_LAYOUT;
  v.setFloat64(L.temperature, o.temperature ?? 0, true);
  v.setFloat64(L.top_p, o.topP ?? 1, true);
  v.setInt32(L.top_k, o.topK ?? 0, true);
  v.setFloat64(L.repetition_penalty, o.repetitionPenalty ?? 1, true);
  let keep: Uint32Array | null = null;
  if (o.penalizedTokenIds) {
    keep = Uint32Array.from(o.penalizedTokenIds);
    v.setBigUint64(L.penalized_ids, BigInt(keep.length ? ptr(keep) : 0), true);
    v.setInt32(L.n_penalized, keep.length, true);
  }
  v.setBigUint64(L.philox_seed, BigInt(o.seed ?? 0), true);
  v.setBigUint64(L.philox_offset, BigInt(offset), true);
  return { bytes: new Uint8Array(buf), keep };
}

export class CudaEngine {
  constructor(readonly h: number, readonly contextLength: number) {}

  runToken(tokenId: number, needLogits: boolean,
           opts: SamplingOptions & { seed?: number; philoxOffset?: number; penalizedTokenIds?: number[] } = {}): number {
    const s = packSampling(opts, opts.philoxOffset ?? 0);
    const out = new Uint32Array(1);
    const rc = S.ck_run_token(this.h, tokenId >>> 0, needLogits ? 1 : 0, ptr(s.bytes), ptr(out));
    check(this.h, rc);
    return out[0];
  }

  prefill(ids: number[], s: PackedSampling): number {
    const a = Uint32Array.from(ids);
    const out = new Uint32Array(1);
    check(this.h, S.ck_prefill(this.h, ptr(a), a.length, 1, ptr(s.bytes), ptr(out)));
    return out[0];
  }

  decode(first: number, maxNew: number, s: PackedSampling, eos: number[]): number[] {
    const e = Uint32Array.from(eos.length ? eos : [0]);
    const out = new Uint32Array(Math.max(1, maxNew));
    const n = new Int32Array(1);
    check(this.h, S.ck_decode(this.h, first >>> 0, maxNew, ptr(s.bytes), ptr(out), eos.length, ptr(e), ptr(n)));
    return Array.from(out.subarray(0, n[0]));
  }

  reset(): void {
    check(this.h, S.ck_reset(this.h));
  }

  // candidates of the sampler: false = the 256-chunk maxima (the reference's),
  // true = the top K of the whole vocabulary (device radix select)
  setExactSampler(exact: boolean): void {
    check(this.h, S.ck_set_sampler(this.h, exact ? 1 : 0));
  }

  get position(): number {
    const p = new Int32Array(1);
    check(this.h, S.ck_position(this.h, ptr(p)));
    return p[0];
  }

  dispose(): void {
    S.ck_destroy(this.h);
  }
}

export interface LoadedLlamaCudaModel {
  runtime: "llama-webgpu";
  def: ModelDef;
  tokenizer: Tokenizer | null;
  engine: CudaEngine;
  ep: "cuda";
  cachedTokenIds: number[];
  cachedNextId: number | null;
}

export async function loadLlamaCudaModel(
  model: ModelDef,
  onProgress?: ProgressCallback,
  onStep?: LoadStepCallback,
): Promise<LoadedLlamaCudaModel> {
  if (model.runtime !== "llama-webgpu") {
    throw new Error(`loadLlamaWgslModel: ${model.id} is not configured for the Llama WGSL runtime`);
  }
  onStep?.({ step: "tokenizer", detail: "loading tokenizer and GGUF header" });
  const tokenizerPromise = model.tokenizer ? Tokenizer.load(model) : Promise.resolve(null);
  const manifest = await buildGgufLlamaManifest(model, onProgress);
  const tokenizer = await tokenizerPromise;
  const contextLength = Math.min(model.maxContext, manifest.model.maxContext);
  onStep?.({ step: "runtime", detail: "opening B200 engine" });
  const hOut = new BigUint64Array(1);
  check(null, S.ck_create(ptr(packCfg(manifest.model, contextLength, model.kvDtype)), 0, ptr(hOut)));
  const h = Number(hOut[0]);
  try {
    for (const [name, spec] of Object.entries(manifest.tensors)) {
      const type = GGML_OF_DTYPE[spec.dtype];
      if (type === undefined) throw new Error(`unsupported tensor dtype ${spec.dtype} for ${name}`);
      if (!spec.external) throw new Error(`Llama WGSL tensor ${name} has no payload`);
      const url = modelFileUrl(model, spec.external.path);
      const bytes = new Uint8Array(await fetchCachedRange(url, spec.external.offset, spec.external.length, onProgress));
      const shape = BigInt64Array.from([...spec.shape].reverse().map((d) => BigInt(d)));   // ggml order
      check(h, S.ck_upload_tensor(h, Buffer.from(name + "\0"), type, ptr(shape), shape.length, ptr(bytes),
                                  bytes.length));
    }
    check(h, S.ck_finalize(h));
  } catch (e) {
    S.ck_destroy(h);
    throw e;
  }
  onStep?.({ step: "ready", detail: "Llama B200 runtime ready" });
  return { runtime: "llama-webgpu", def: model, tokenizer, engine: new CudaEngine(h, contextLength), ep: "cuda",
           cachedTokenIds: [], cachedNextId: null };
}

export interface GenerateLlamaCudaOptions {
  maxNewTokens?: number;
  temperature?: number;
  topP?: number;
  topK?: number;
  repetitionPenalty?: number;
  seed?: number;   // Philox key: the draws replace Math.random
  sampler?: "chunk" | "exact";   // candidate list (an extension; "chunk" is the reference's)
  onToken?: (info: { id: number; text: string; cumulative: string }) => void;
  shouldStop?: () => boolean;
}

function commonPrefixLength(a: number[], b: number[]): number {
  const n = Math.min(a.length, b.length);
  let i = 0;
  while (i < n && a[i] === b[i]) i++;
  return i;
}

// generateLlamaWgsl (:242-314) step for step: prefix reuse, prompt suffix
// through ck_prefill, then the device decode loop (ck_decode) or, when the
// caller watches every token, one ck_run_token per id.
export async function generateLlamaCuda(
  loaded: LoadedLlamaCudaModel,
  promptIds: number[],
  opts: GenerateLlamaCudaOptions = {},
): Promise<{ text: string; ids: number[]; tokensPerSec: number }> {
  const d = loaded.def;
  const eng = loaded.engine;
  const mx = Math.min(opts.maxNewTokens ?? 128, d.maxContext - promptIds.length);
  const eos = new Set(d.eosIds);
  const sampling: SamplingOptions = {
    temperature: opts.temperature ?? 0,
    topP: opts.topP ?? 1,
    topK: opts.topK ?? 0,
    repetitionPenalty: opts.repetitionPenalty ?? d.defaultRepetitionPenalty ?? 1,
  };
  const sampled = needsSamplingReadback(sampling);
  eng.setExactSampler(opts.sampler === "exact");
  let draws = 0;
  const mk = () => packSampling({ ...sampling, seed: opts.seed ?? 0 }, draws);
  const decodeText = (ids: number[]) => (loaded.tokenizer ? loaded.tokenizer.decode(ids) : "");

  const t0 = performance.now();
  let prefixLen = commonPrefixLength(loaded.cachedTokenIds, promptIds);
  if (prefixLen !== loaded.cachedTokenIds.length) {
    eng.reset();
    loaded.cachedTokenIds = [];
    loaded.cachedNextId = null;
    prefixLen = 0;
  }
  let nextId = 0;
  const suffix = promptIds.slice(prefixLen);
  if (suffix.length === 0 && loaded.cachedNextId !== null) {
    nextId = loaded.cachedNextId;
  } else if (suffix.length > 0) {
    nextId = eng.prefill(suffix, mk());
    if (sampled) draws++;
  }

  let generated: number[] = [];
  let cumulative = "";
  if (mx > 0 && !opts.onToken && !opts.shouldStop) {
    generated = eng.decode(nextId, mx, mk(), [...eos]);
    if (generated.length) nextId = generated[generated.length - 1];
    cumulative = decodeText(generated);
  } else {
    for (let step = 0; step < mx; step++) {
      if (opts.shouldStop?.()) break;
      generated.push(nextId);
      const full = decodeText(generated);
      const piece = full.slice(cumulative.length);
      cumulative = full;
      opts.onToken?.({ id: nextId, text: piece, cumulative });
      if (eos.has(nextId) || step + 1 >= mx) break;
      const s = mk();
      const out = new Uint32Array(1);
      check(eng.h, S.ck_run_token(eng.h, nextId >>> 0, 1, ptr(s.bytes), ptr(out)));
      nextId = out[0];
      if (sampled) draws++;
    }
  }
  loaded.cachedTokenIds = [...promptIds, ...generated];
  const last = generated.length ? generated[generated.length - 1] : -1;
  loaded.cachedNextId = eos.has(last) ? null : nextId;
  const elapsed = (performance.now() - t0) / 1000;
  return { text: cumulative, ids: generated, tokensPerSec: generated.length / Math.max(elapsed, 1e-3) };
}

export function disposeLlamaCuda(loaded: LoadedLlamaCudaModel): void {
  loaded.engine.dispose();
}

export function resetLlamaCudaConversation(loaded: LoadedLlamaCudaModel): void {
  loaded.engine.reset();
  loaded.cachedTokenIds = [];
  loaded.cachedNextId = null;
}

export { CK_ECONTEXT };
