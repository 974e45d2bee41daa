// CudaBackend — textsift's InferenceBackend on a B200 (sm_100a) through the
// N-API addon textsift_cuda.node (textsift_cuda_napi.c beside this file),
// which links libtextsift_cuda.so.
//
// It is written to sit at packages/textsift/src/native/cuda-backend.ts, next
// to the reference's NodeBackend (native/backend.ts:361-759), and to take the
// same BackendConstructionOptions.  Differences from NodeBackend, on purpose:
// the addon reads and converts the ONNX initializers itself (the rules of
// loadOnnxWeights, browser/backends/wasm.ts:328-453), owns every device
// buffer and runs the whole dispatch sequence in one call, so this class only
// fetches the two model files and passes token ids.  forwardPackedTags()
// additionally serves redactBatch: many chunks in one launch with the BIOES
// Viterbi decode on the GPU (browser/privacy-filter.ts:264-293, 497-500).
//
// Node is not installed where this repository is built, so this file is not
// compiled or run there; tests/test_node_binding.py checks that it calls only
// what the addon registers.

import { createRequire } from "node:module";
import { fileURLToPath } from "node:url";
import { dirname, resolve } from "node:path";
import type { InferenceBackend, Logits, BackendConstructionOptions } from "../browser/backends/abstract.js";
import { fetchOnnxGraph, fetchOnnxExtData } from "./loader.js";

/** What textsift_cuda.node exports (textsift_cuda_napi.c, Init). */
export interface CudaApi {
  cudaCreateBackend(device?: number, maxTokens?: number, maxSeqLen?: number): bigint;
  cudaDestroyBackend(handle: bigint): void;
  cudaDeviceName(handle: bigint): string;
  cudaLoadOnnx(handle: bigint, graph: Uint8Array, extData: Uint8Array | null): void;
  cudaLoadTensor(handle: bigint, name: string, dtype: number, bytes: Uint8Array): void;
  cudaFinalize(handle: bigint): void;
  cudaForwardPacked(handle: bigint, ids: Int32Array, mask: Uint8Array | null, offsets: Uint32Array): Float32Array;
  cudaForwardPackedTags(handle: bigint, ids: Int32Array, mask: Uint8Array | null, offsets: Uint32Array,
                        calibration: Float32Array): Uint8Array;
  tokCreate(tokenizerJson: Uint8Array): bigint;
  tokDestroy(tok: bigint): void;
  tokEncode(tok: bigint, utf8: Uint8Array): { ids: Int32Array; charOffsets: Uint32Array };
}

const NUM_CLASSES = 33;

/** The addon path: TEXTSIFT_CUDA_ADDON, else textsift_cuda.node beside this file. */
function addonPath(): string {
  const env = process.env.TEXTSIFT_CUDA_ADDON;
  if (env) return env;
  return resolve(dirname(fileURLToPath(import.meta.url)), "textsift_cuda.node");
}

export function loadCudaApi(): CudaApi {
  return createRequire(import.meta.url)(addonPath()) as CudaApi;
}

export class CudaBackend implements InferenceBackend {
  readonly name = "cuda";
  private api: CudaApi;
  private handle: bigint = 0n;
  private opts: BackendConstructionOptions;
  private device: number;

  constructor(opts: BackendConstructionOptions, device = 0, api: CudaApi = loadCudaApi()) {
    this.opts = opts;
    this.device = device;
    this.api = api;
  }

  async warmup(): Promise<void> {
    if (this.handle !== 0n) return; // idempotent: the base PrivacyFilter calls it twice (backend.ts:408)
    const loaderOpts = {
      cacheDir: this.opts.cacheDir,
      modelPath: this.opts.modelPath,
      offline: this.opts.offline,
    };
    const [graph, ext] = await Promise.all([
      fetchOnnxGraph(this.opts.bundle.modelSource, loaderOpts),
      fetchOnnxExtData(this.opts.bundle.modelSource, loaderOpts),
    ]);
    const h = this.api.cudaCreateBackend(this.device);
    try {
      this.api.cudaLoadOnnx(h, graph, ext);
      this.api.cudaFinalize(h);
    } catch (e) {
      this.api.cudaDestroyBackend(h);
      throw e;
    }
    this.handle = h;
  }

  async forward(tokenIds: Int32Array, attentionMask: Uint8Array): Promise<Logits> {
    if (this.handle === 0n) throw new Error("CudaBackend: call warmup() before forward()");
    if (attentionMask.length !== tokenIds.length) {
      throw new Error(
        `CudaBackend.forward: attentionMask length ${attentionMask.length} != tokenIds length ${tokenIds.length}`,
      );
    }
    const offsets = Uint32Array.of(0, tokenIds.length);
    const data = tokenIds.length === 0
      ? new Float32Array(0)
      : this.api.cudaForwardPacked(this.handle, tokenIds, attentionMask, offsets);
    return { data, sequenceLength: tokenIds.length, numClasses: NUM_CLASSES };
  }

  /** Many chunks (e.g. every chunk of a redactBatch call) in one launch,
   *  decoded to BIOES tags on the GPU with the decoder's calibration (the six
   *  ViterbiCalibration fields in declaration order, model/calibration.ts:29-36).
   *  Returns one tag array per chunk, as ViterbiDecoder.decode would. */
  forwardPackedTags(chunks: Int32Array[], calibration: Float32Array, masks?: Uint8Array[]): Uint8Array[] {
    if (this.handle === 0n) throw new Error("CudaBackend: call warmup() before forwardPackedTags()");
    const offsets = new Uint32Array(chunks.length + 1);
    for (let i = 0; i < chunks.length; i++) offsets[i + 1] = offsets[i] + chunks[i].length;
    const total = offsets[chunks.length];
    const ids = new Int32Array(total);
    chunks.forEach((c, i) => ids.set(c, offsets[i]));
    let mask: Uint8Array | null = null;
    if (masks) {
      mask = new Uint8Array(total);
      masks.forEach((m, i) => mask!.set(m, offsets[i]));
    }
    const tags = total === 0 ? new Uint8Array(0)
      : this.api.cudaForwardPackedTags(this.handle, ids, mask, offsets, calibration);
    return chunks.map((_, i) => tags.subarray(offsets[i], offsets[i + 1]));
  }

  dispose(): void {
    if (this.handle !== 0n) {
      this.api.cudaDestroyBackend(this.handle);
      this.handle = 0n;
    }
  }
}

/** For resolveAuto (packages/textsift/src/index.ts:70-95): try the CUDA
 *  backend before NodeBackend; null when there is no usable B200 or no addon,
 *  so the resolver falls through to its existing native / WASM choice. */
export async function tryCudaBackend(opts: BackendConstructionOptions): Promise<CudaBackend | null> {
  try {
    const backend = new CudaBackend(opts);
    await backend.warmup();
    return backend;
  } catch {
    return null;
  }
}
