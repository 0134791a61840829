//! `Model` and `ModelTiles` (`kernels/src/model.rs:89-450`) over libqne.so.

use std::collections::BTreeMap;
use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};
use std::ptr;
use std::sync::Mutex;

use crate::ffi;
use crate::{check, Error, ErrorKind, Result, Tile};

/// GEMV kernel per matrix kind (`kernels/src/model.rs:89-99`). Accepted and validated with the
/// reference's rules; the CUDA kernels choose their own shapes.
#[derive(Clone, Copy, Debug)]
#[cfg_attr(feature = "serde", derive(serde::Serialize, serde::Deserialize))]
pub struct ModelTiles {
    pub gdn_in: Tile,
    pub attn_in: Tile,
    pub out: Tile,
    pub gate_up: Tile,
    pub down: Tile,
    pub lm_head: Tile,
}

/// One row of the reference's tuning report (`kernels/src/lib.rs`, `GemvTiming`).
#[derive(Clone, Debug)]
pub struct GemvTiming {
    pub name: String,
    pub rows: u32,
    pub k: u32,
    pub tile: Tile,
    pub ms: f64,
}

impl ModelTiles {
    fn all(&self) -> [(&'static str, Tile); 6] {
        [
            ("gdn_in", self.gdn_in),
            ("attn_in", self.attn_in),
            ("out", self.out),
            ("gate_up", self.gate_up),
            ("down", self.down),
            ("lm_head", self.lm_head),
        ]
    }

    /// The profile as the reference serializes it (serde field names).
    pub fn to_json(&self) -> String {
        let parts: Vec<String> = self
            .all()
            .iter()
            .map(|(n, t)| {
                format!(
                    "\"{n}\":{{\"f16\":{},\"tpr\":{},\"rpw\":{},\"rpt\":{},\"splits\":{}}}",
                    t.f16, t.tpr, t.rpw, t.rpt, t.splits
                )
            })
            .collect();
        format!("{{{}}}", parts.join(","))
    }

    /// `ModelTiles::validate` (`kernels/src/model.rs:101-109`): every tile within the reference's
    /// dispatch geometry; otherwise "invalid kernel tile profile: ...".
    pub fn validate(&self) -> Result<()> {
        let json = self.to_json();
        // SAFETY: pointer and length of a live byte buffer.
        check(unsafe { ffi::qne_validate_tiles(json.as_ptr() as *const c_char, json.len()) })
    }

    /// The plain f32 kernel everywhere (`kernels/src/model.rs:110-114`).
    pub fn f32() -> Self {
        let t = Tile { f16: false, tpr: 16, rpw: 4, rpt: 1, splits: 1 };
        Self { gdn_in: t, attn_in: t, out: t, gate_up: t, down: t, lm_head: t }
    }

    /// The reference's default profile (`kernels/src/model.rs:139-144`).
    pub fn fast() -> Self {
        let f16 = |tpr, rpw, rpt, splits| Tile { f16: true, tpr, rpw, rpt, splits };
        let f32 = Tile { f16: false, tpr: 16, rpw: 4, rpt: 1, splits: 1 };
        Self {
            gdn_in: f16(16, 4, 4, 1),
            attn_in: f16(4, 32, 4, 1),
            out: f32,
            gate_up: f16(4, 16, 4, 1),
            down: f32,
            lm_head: f16(4, 32, 4, 1),
        }
    }

    /// `ModelTiles::tune` (`kernels/src/model.rs:116-137`): the CUDA kernels have no tile knob to
    /// search, so this checks the shape as the reference does and returns the default profile
    /// with an empty report.
    pub async fn tune(index_json: &str, _dxc: Option<&str>, log: &dyn Fn(&str)) -> Result<(Self, Vec<GemvTiming>)> {
        let hidden = config_field(index_json, "hidden").unwrap_or(0);
        let inter = match config_field(index_json, "intermediate") {
            Some(v) if v != 0 => v,
            _ if hidden == 1024 => 3584,
            _ => 6144,
        };
        if !matches!((hidden, inter), (1024, 3584) | (2048, 6144)) {
            return Err(Error { kind: ErrorKind::Format, message: "unsupported tuning shape".into() });
        }
        log("tuning skipped: the CUDA kernels choose their own shapes");
        Ok((Self::fast(), Vec::new()))
    }
}

/// The integer value of `"key": <n>` inside index.json's config object (enough for `tune`; the
/// full parse and validation happen in the library at load).
fn config_field(index_json: &str, key: &str) -> Option<u64> {
    let cfg = &index_json[index_json.find("\"config\"")?..];
    let at = cfg.find(&format!("\"{key}\""))? + key.len() + 2;
    let rest = cfg[at..].trim_start().strip_prefix(':')?.trim_start();
    let digits: String = rest.chars().take_while(|c| c.is_ascii_digit()).collect();
    digits.parse().ok()
}

/// Engine options of `Model::load_with` (no counterpart in the reference).
#[derive(Clone, Copy, Debug, Default)]
pub struct LoadOptions {
    /// CUDA device ordinal.
    pub device: i32,
    /// Also accept architectures other than Qwen3.5-0.8B / -2B (`QNE_LOAD_ANY_SHAPE`).
    pub any_shape: bool,
}

struct Handle(*mut ffi::qne_model);

// SAFETY: the handle is only used under the Mutex below, one call at a time, which is what the
// library requires (one host thread at a time per model).
unsafe impl Send for Handle {}

/// A loaded decoder on one GPU (`kernels/src/model.rs:147-450`).
pub struct Model {
    raw: Mutex<Handle>,
    vocab: usize,
    pub adapter: String,
}

impl Drop for Model {
    fn drop(&mut self) {
        let h = self.raw.get_mut().map(|h| h.0).unwrap_or(ptr::null_mut());
        if !h.is_null() {
            // SAFETY: the handle came from qne_model_load and is freed once.
            unsafe { ffi::qne_model_free(h) };
        }
    }
}

impl Model {
    /// `Model::load` (`kernels/src/model.rs:171`): validates index.json against the weights as
    /// `Index::validate` does, copies the weights to the device (the caller may drop its copy
    /// afterwards) and builds the decode graphs. `allow_f16` and `dxc` select wgpu shader paths
    /// and mean nothing on CUDA; `tiles` is validated.
    pub async fn load(
        index_json: &str,
        weights: &[u8],
        tiles: ModelTiles,
        _allow_f16: bool,
        _dxc: Option<&str>,
    ) -> Result<Self> {
        tiles.validate()?;
        Self::load_with(index_json, weights, LoadOptions::default())
    }

    /// `load` on a chosen device, optionally accepting any supported shape.
    pub fn load_with(index_json: &str, weights: &[u8], opts: LoadOptions) -> Result<Self> {
        let mut h: *mut ffi::qne_model = ptr::null_mut();
        let flags = if opts.any_shape { ffi::QNE_LOAD_ANY_SHAPE } else { 0 };
        // SAFETY: pointers and lengths of live buffers; `h` receives the handle.
        check(unsafe {
            ffi::qne_model_load_ex(
                index_json.as_ptr() as *const c_char,
                index_json.len(),
                weights.as_ptr() as *const c_void,
                weights.len(),
                opts.device as c_int,
                flags,
                &mut h,
            )
        })?;
        let mut info = ffi::qne_model_info::default();
        // SAFETY: `h` is a valid handle.
        let st = unsafe { ffi::qne_model_info_get(h, &mut info) };
        // SAFETY: as above; the adapter string lives as long as the model and is copied.
        let adapter = unsafe { CStr::from_ptr(ffi::qne_adapter(h)) }.to_string_lossy().into_owned();
        let model = Model { raw: Mutex::new(Handle(h)), vocab: info.vocab.max(0) as usize, adapter };
        check(st)?;
        Ok(model)
    }

    fn with<T>(&self, f: impl FnOnce(*mut ffi::qne_model) -> Result<T>) -> Result<T> {
        let guard = self.raw.lock().unwrap_or_else(|p| p.into_inner());
        f(guard.0)
    }

    /// `Model::profile_token` (`kernels/src/model.rs:305-307`): consumes one greedy token;
    /// milliseconds per dispatch label, each kernel timed alone. Diagnostic only.
    pub async fn profile_token(&self) -> Result<BTreeMap<String, f64>> {
        self.with(|h| {
            let mut n = 0usize;
            let mut buf = vec![ffi::qne_profile_entry { label: [0; 48], ms: 0.0, dispatches: 0, pad: 0 }; 64];
            // SAFETY: `buf` holds `cap` entries.
            check(unsafe { ffi::qne_profile_token(h, buf.as_mut_ptr(), buf.len(), &mut n) })?;
            let mut out = BTreeMap::new();
            for e in buf.iter().take(n.min(buf.len())) {
                // SAFETY: labels are NUL-terminated within their 48 bytes.
                let label = unsafe { CStr::from_ptr(e.label.as_ptr()) }.to_string_lossy().into_owned();
                out.insert(label, e.ms);
            }
            Ok(out)
        })
    }

    /// `Model::dispatches_per_token` (`kernels/src/model.rs:309`).
    pub fn dispatches_per_token(&self) -> usize {
        self.with(|h| Ok(unsafe { ffi::qne_dispatches_per_token(h) })).unwrap_or(0)
    }

    /// `Model::reset` (`kernels/src/model.rs:314`): clears the recurrent states and the KV cache.
    /// Like the reference it returns nothing; a device failure surfaces on the next call.
    pub fn reset(&self) {
        let _ = self.with(|h| check(unsafe { ffi::qne_reset(h) }));
    }

    /// `Model::prefill` (`kernels/src/model.rs:324`): the prompt from position 0, one token per
    /// step; afterwards `logits` and `last_token` describe the prediction after the last id.
    pub async fn prefill(&self, ids: &[u32]) -> Result<()> {
        let n = u32::try_from(ids.len()).map_err(|_| too_long())?;
        self.with(|h| check(unsafe { ffi::qne_prefill(h, ids.as_ptr(), n) }))
    }

    /// `Model::prefill_batched` (`kernels/src/model.rs:339`).
    pub async fn prefill_batched(&self, ids: &[u32]) -> Result<()> {
        self.prefill_chunk(ids, 0, true).await
    }

    /// `Model::prefill_from` (`kernels/src/model.rs:344`).
    pub async fn prefill_from(&self, ids: &[u32], start: u32) -> Result<()> {
        self.prefill_chunk(ids, start, true).await
    }

    /// `Model::prefill_chunk` (`kernels/src/model.rs:349`): `ids` at positions start.., in batched
    /// chunks; with `finish_logits` the logits after the last id and its greedy pick.
    pub async fn prefill_chunk(&self, ids: &[u32], start: u32, finish_logits: bool) -> Result<()> {
        let n = u32::try_from(ids.len()).map_err(|_| too_long())?;
        self.with(|h| check(unsafe { ffi::qne_prefill_chunk(h, ids.as_ptr(), n, start, finish_logits as c_int) }))
    }

    /// `Model::logits` (`kernels/src/model.rs:374`).
    pub async fn logits(&self) -> Result<Vec<f32>> {
        let mut out = vec![0f32; self.vocab];
        self.with(|h| check(unsafe { ffi::qne_logits(h, out.as_mut_ptr(), out.len()) }))?;
        Ok(out)
    }

    /// `Model::step` (`kernels/src/model.rs:380`): feeds `token` at `pos`, returns the logits.
    pub async fn step(&self, token: u32, pos: u32) -> Result<Vec<f32>> {
        let mut out = vec![0f32; self.vocab];
        self.with(|h| check(unsafe { ffi::qne_step(h, token, pos, out.as_mut_ptr(), out.len()) }))?;
        Ok(out)
    }

    /// `Model::snapshot` (`kernels/src/model.rs:395`).
    pub fn snapshot(&self) {
        let _ = self.with(|h| check(unsafe { ffi::qne_snapshot(h) }));
    }

    /// `Model::restore` (`kernels/src/model.rs:406`): "no snapshot taken" without a snapshot.
    pub fn restore(&self) -> Result<()> {
        self.with(|h| check(unsafe { ffi::qne_restore(h) }))
    }

    /// `Model::last_token` (`kernels/src/model.rs:417`): the greedy pick and the next position.
    pub async fn last_token(&self) -> Result<(u32, u32)> {
        let (mut t, mut p) = (0u32, 0u32);
        self.with(|h| check(unsafe { ffi::qne_last_token(h, &mut t, &mut p) }))?;
        Ok((t, p))
    }

    /// `Model::decode` (`kernels/src/model.rs:426`): greedy decoding, `window` tokens per host
    /// sync (ids inside larger windows are `u32::MAX`), stopping after a stop id.
    pub async fn decode(&self, n: usize, window: u32, stop: &[u32]) -> Result<Vec<u32>> {
        let n32 = u32::try_from(n).map_err(|_| too_long())?;
        let mut out = vec![0u32; n.max(1)];
        let mut got = 0u32;
        self.with(|h| {
            check(unsafe {
                ffi::qne_decode(h, n32, window, stop.as_ptr(), stop.len() as u32, out.as_mut_ptr(), &mut got)
            })
        })?;
        out.truncate(got as usize);
        Ok(out)
    }

    /// One step and a draw on the device (`qne_step_sample`; no counterpart in the reference,
    /// whose agent samples on the host after reading the logits back).
    pub fn step_sample(
        &self,
        sampler: &DeviceSampler,
        token: u32,
        pos: u32,
        mask: Option<&[u32]>,
        mask_tokens: u32,
        bias: Option<(u32, f32)>,
    ) -> Result<u32> {
        let mut out = 0u32;
        let (bias_token, bias) = bias.map(|(t, b)| (t as i32, b)).unwrap_or((-1, 0.0));
        let mask_ptr = mask.map(|m| m.as_ptr()).unwrap_or(ptr::null());
        let s = sampler.raw;
        self.with(|h| {
            check(unsafe { ffi::qne_step_sample(h, s, token, pos, mask_ptr, mask_tokens, bias_token, bias, &mut out) })
        })?;
        Ok(out)
    }
}

/// A device-side sampler of one generation (`qne_sampler_*`): temperature, top-k, top-p and
/// presence penalty as `Sampler::try_sample` (`src/sampling.rs:58-67`). Free it before its model.
pub struct DeviceSampler {
    raw: *mut ffi::qne_sampler,
}

impl DeviceSampler {
    pub fn new(model: &Model, temperature: f32, top_k: u32, top_p: f32, seed: u64, presence_penalty: f32) -> Result<Self> {
        let opts = ffi::qne_sampling { temperature, top_k, top_p, seed, presence_penalty };
        let mut raw = ptr::null_mut();
        model.with(|h| check(unsafe { ffi::qne_sampler_create(h, &opts, &mut raw) }))?;
        Ok(Self { raw })
    }
}

impl Drop for DeviceSampler {
    fn drop(&mut self) {
        // SAFETY: created by qne_sampler_create, freed once.
        unsafe { ffi::qne_sampler_free(self.raw) };
    }
}

fn too_long() -> Error {
    Error { kind: ErrorKind::ContextLimit, message: "context limit of 4096 tokens reached".into() }
}
