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

/** pickToken on the GPU: one row, the reference's penalty and draw rules. */
export function pickTokenCuda(lastLogits, generated, inputIds, opts) {
  const a = loadCudaSampler();
  let hist = null, off = null;
  if (generated.length) {
    hist = Int32Array.from(inputIds.concat(generated), (v) => (Number.isInteger(v) && v >= 0 && v < 2 ** 31 ? v : -1));
    off = Int32Array.of(0, hist.length);
  }
  const greedy = !opts.doSample || opts.temperature <= 0.0001;
  const u = greedy ? null : Float64Array.of(Math.random());
  const logits = lastLogits instanceof Float32Array ? lastLogits : Float32Array.from(lastLogits);
  const ids = a.sample(logits, 1, logits.length, hist, off, opts, u);
  return [ids[0], true];
}
