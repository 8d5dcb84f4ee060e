/**
 * sampler.ts over the B200 sampler: the surface of xOAviOx/tabby src/engine/sampler.ts
 * (SamplingParams :83-91, DEFAULT_SAMPLING :93-98, SeededRandom :105-119, SampleOutcome
 * :121-135, sampleFromTopK :147-212) with the GPU work done by libtabbysample.so through the
 * zero-dependency N-API addon native/tabby_napi.c. Not built in this repository's images
 * (Node.js is absent); a maintainer drops it next to the reference's sampler and builds
 * the addon with native/binding.gyp.
 *
 * Draws follow the reference exactly: sampleFromTopK calls random.next() only when it
 * samples (temperature > 0, after the empty-set throw and the greedy return), so one
 * SeededRandom shared across calls replays the reference's token stream.
 */
// eslint-disable-next-line @typescript-eslint/no-var-requires
const native = require('../native/build/Release/tabby_napi.node');

export interface SamplingParams {
  temperature: number;
  topK: number;
  topP: number;
  seed: number;
}

export const DEFAULT_SAMPLING: SamplingParams = { temperature: 0.7, topK: 40, topP: 0.9, seed: 0 };

export interface SampleOutcome {
  id: number;
  probability: number;
  consideredCount: number;
  poolMass: number;
  poolExhausted: boolean;
}

export interface TopKResult {
  maxLogit: number;
  sumExp: number;
  ids: number[];
  logits: number[];
}

/** mulberry32, as sampler.ts:105-119. */
export class SeededRandom {
  private state: number;

  constructor(seed: number) {
    this.state = seed >>> 0;
  }

  next(): number {
    this.state = (this.state + 0x6d2b79f5) >>> 0;
    let t = this.state;
    t = Math.imul(t ^ (t >>> 15), t | 1);
    t ^= t + Math.imul(t ^ (t >>> 7), t | 61);
    return ((t ^ (t >>> 14)) >>> 0) / 4294967296;
  }
}

const OUT_FIELDS = 6;

function outcomeAt(outcomes: Float64Array, r: number): SampleOutcome {
  const o = OUT_FIELDS * r;
  return {
    id: outcomes[o],
    probability: outcomes[o + 1],
    consideredCount: outcomes[o + 2],
    poolMass: outcomes[o + 3],
    poolExhausted: outcomes[o + 4] !== 0,
  };
}

/** One handle per worker thread (the reference's worker owns the device). */
export class Sampler {
  private readonly handle: unknown;

  constructor(opts: { device?: number; maxTopK?: number; maxRows?: number; maxVocab?: number } = {}) {
    this.handle = native.create(opts);
  }

  /**
   * sample(logits, {temperature, topK, topP}, rng) -> token id: pool rule, max, sum-exp,
   * exact top-k and sampleFromTopK on the GPU for one row.
   */
  sample(logits: Float32Array, params: SamplingParams, random: SeededRandom): number {
    return this.sampleBatch(logits, 1, logits.length, [params], random)[0].id;
  }

  /**
   * Rows of `vocab` logits, one SamplingParams for all rows or one per row; the uniforms
   * are drawn from `random` in row order, only for rows that sample (temperature > 0).
   */
  sampleBatch(logits: Float32Array, rows: number, vocab: number,
              params: SamplingParams[] | SamplingParams, random: SeededRandom): SampleOutcome[] {
    const [p, u] = this.packRows(rows, params, random);
    const res = native.sampleBatch(this.handle, logits, rows, vocab, p, u);
    return Array.from({ length: rows }, (_, r) => outcomeAt(res.outcomes, r));
  }

  /** sampleBatch on a libuv worker thread. */
  async sampleBatchAsync(logits: Float32Array, rows: number, vocab: number,
                         params: SamplingParams[] | SamplingParams,
                         random: SeededRandom): Promise<SampleOutcome[]> {
    const [p, u] = this.packRows(rows, params, random);
    const res = await native.sampleBatchAsync(this.handle, logits, rows, vocab, p, u);
    return Array.from({ length: rows }, (_, r) => outcomeAt(res.outcomes, r));
  }

  private packRows(rows: number, params: SamplingParams[] | SamplingParams,
                   random: SeededRandom): [Float64Array, Float64Array] {
    const list = Array.isArray(params) ? params : Array(rows).fill(params);
    if (list.length !== rows) throw new RangeError(`${list.length} SamplingParams for ${rows} rows`);
    const p = new Float64Array(3 * rows);
    const u = new Float64Array(rows);
    for (let r = 0; r < rows; r++) {
      p[3 * r] = list[r].temperature;
      p[3 * r + 1] = list[r].topK;
      p[3 * r + 2] = list[r].topP;
      u[r] = list[r].temperature > 0 ? random.next() : 0;
    }
    return [p, u];
  }
}

/**
 * sampleFromTopK(top, params, random) (sampler.ts:147-212) in the library's float64
 * arithmetic, for callers that already hold a TopKResult.
 */
export function sampleFromTopK(top: TopKResult, params: SamplingParams,
                               random: SeededRandom): SampleOutcome {
  if (top.ids.length === 0) throw new Error('sampleFromTopK: empty candidate set');
  const u = params.temperature > 0 ? random.next() : 0;
  const o: Float64Array = native.sampleFromTopK(Int32Array.from(top.ids),
                                                Float32Array.from(top.logits), top.maxLogit,
                                                top.sumExp, params.temperature, params.topP, u);
  return { id: o[0], probability: o[1], consideredCount: o[2], poolMass: o[3],
           poolExhausted: o[4] !== 0 };
}

/** Pool size of the worker (inference.worker.ts:120-123). */
export function poolSize(temperature: number, topK: number, maxTopK = 64): number {
  return native.poolSize(temperature, topK, maxTopK);
}
