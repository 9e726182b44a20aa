/**
 * mini.js 'cuda' sampler backend: a lazy, Node-only loader for the
 * libminisample N-API addon, plus the pickToken replacement that calls it.
 *
 * Drop-in for src/generation.js:71-81.  Same arguments, same result
 * ([tokenId, true]), same option semantics (normalizeOptions,
 * src/generation.js:57-68), one Math.random() per sampled step and none when
 * greedy (src/generation.js:43,76).  Failures throw; there is no JS fallback.
 *
 * The addon is loaded inside a function (process.dlopen), never by a static
 * import, so the regex bundler (build.mjs:41-71) never sees it.
 */

let addon = null;

export function loadCudaSampler(path) {
  if (addon) return addon;
  if (typeof process === 'undefined' || !process.versions || !process.versions.node) {
    throw new Error("[mini.js] the 'cuda' sampler backend needs Node.js");
  }
  const file = path || process.env.MINISAMPLE_ADDON || new URL('../minisample/minisample.node', import.meta.url).pathname;
  const mod = { exports: {} };
  process.dlopen(mod, file);
  addon = mod.exports;
  return addon;
}

// Ids that can never index the vocabulary become -1, which the penalty ignores.
const histId = (v) => (Number.isInteger(v) && v >= 0 && v < 2 ** 31 ? v : -1);
const isGreedy = (opts) => !opts.doSample || opts.temperature <= 0.0001;

/** The addon's arguments for one row (src/generation.js:72-79): the penalty
 * history only once something was generated, one Math.random() when sampled. */
function rowArgs(lastLogits, generated, inputIds, opts) {
  let hist = null, off = null;
  if (generated.length) {
    hist = Int32Array.from(inputIds.concat(generated), histId);
    off = Int32Array.of(0, hist.length);
  }
  const u = isGreedy(opts) ? null : Float64Array.of(Math.random());
  const logits = lastLogits instanceof Float32Array ? lastLogits : Float32Array.from(lastLogits);
  return [logits, 1, logits.length, hist, off, opts, u];
}

/** pickToken on the GPU: one row, the reference's penalty and draw rules. */
export function pickTokenCuda(lastLogits, generated, inputIds, opts) {
  const ids = loadCudaSampler().sample(...rowArgs(lastLogits, generated, inputIds, opts));
  return [ids[0], true];
}

/** pickTokenCuda on a libuv worker thread, for generateAsync
 * (src/generation.js:121-142): the uniform is drawn when it is called, so the
 * Math.random() sequence is the synchronous one; resolves to [tokenId, true]. */
export async function pickTokenCudaAsync(lastLogits, generated, inputIds, opts) {
  const ids = await loadCudaSampler().sampleAsync(...rowArgs(lastLogits, generated, inputIds, opts));
  return [ids[0], true];
}

/**
 * One sampler call over B rows for batched generation: row i is
 * pickToken(rows[i], generatedRows[i], inputIdsRows[i], opts) with its own
 * penalty history (CSR: one Int32Array, B+1 offsets; empty until row i
 * generated something) and one Math.random() per row, drawn in row order,
 * when sampling.  `rows` is B Float32Arrays of V logits, or one Float32Array of
 * B*V.  Returns the B ids as an Int32Array.
 */
export function sampleRowsCuda(rows, generatedRows, inputIdsRows, opts) {
  const B = generatedRows.length;
  let logits;
  if (rows instanceof Float32Array) {
    logits = rows;
  } else {
    logits = new Float32Array(B * rows[0].length);
    rows.forEach((r, i) => logits.set(r, i * rows[0].length));
  }
  const V = logits.length / B;
  const off = new Int32Array(B + 1);
  for (let i = 0; i < B; i++) {
    const g = generatedRows[i].length;
    off[i + 1] = off[i] + (g ? inputIdsRows[i].length + g : 0);
  }
  const hist = new Int32Array(off[B]);
  for (let i = 0; i < B; i++) {
    if (!generatedRows[i].length) continue;
    let k = off[i];
    for (const v of inputIdsRows[i]) hist[k++] = histId(v);
    for (const v of generatedRows[i]) hist[k++] = histId(v);
  }
  let u = null;
  if (!isGreedy(opts)) {
    u = new Float64Array(B);
    for (let i = 0; i < B; i++) u[i] = Math.random();
  }
  return loadCudaSampler().sample(logits, B, V, off[B] ? hist : null, off[B] ? off : null, opts, u);
}
