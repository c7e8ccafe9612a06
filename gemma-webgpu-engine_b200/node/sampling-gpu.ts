// sampleToken on the B200: the same signature and behaviour as the reference's
// src/runtime/sampling.ts:18-65, for its call sites in src/runtime/gemma-session.ts
// (686, 705, 1328).  The logits that the reference reads back as a Float32Array are
// sampled by libgsampler through the Node-API addon (gsampler_napi.cc, built by
// `node-gyp rebuild` in this folder).
//
// What stays on the host, as in the reference: the repetition window
// (history.slice(-repetitionWindow)), counted into a Map in first-occurrence order (the
// counting sampleToken does itself, sampling.ts:21-24), and the call of `random()`, made
// exactly once and only when temperature != 0, so the caller's SeededRandom advances as
// it would.
import { createRequire } from "node:module";

// The DecodingConfig fields sampleToken reads (src/runtime/decoding.ts:1-14); the
// reference's own DecodingConfig is assignable to it.
export interface DecodingConfig {
  temperature: number;
  topK: number;
  topP: number;
  minP: number;
  typicalP: number;
  repetitionPenalty: number;
  repetitionWindow: number;
  presencePenalty: number;
  frequencyPenalty: number;
}

interface GsamplerAddon {
  sampleHost(
    logits: Float32Array,
    historyIds: Int32Array,
    historyCounts: Int32Array,
    config: DecodingConfig,
    uniform: number,
    softcap?: number,
  ): number;
}

const addon = createRequire(import.meta.url)("./build/Release/gsampler.node") as GsamplerAddon;

export function sampleToken(
  rawLogits: ArrayLike<number>,
  history: readonly number[],
  config: DecodingConfig,
  random: () => number,
): number {
  if (rawLogits.length === 0) throw new Error("Cannot sample empty logits");
  const logits = rawLogits instanceof Float32Array ? rawLogits : Float32Array.from(rawLogits);
  const recent = config.repetitionWindow === 0 ? [] : history.slice(-config.repetitionWindow);
  const counts = new Map<number, number>();
  for (const token of recent) counts.set(token, (counts.get(token) ?? 0) + 1);
  const ids = Int32Array.from(counts.keys());
  const occurrences = Int32Array.from(counts.values());
  const uniform = config.temperature === 0 ? 0 : random();
  return addon.sampleHost(logits, ids, occurrences, config, uniform);
}
