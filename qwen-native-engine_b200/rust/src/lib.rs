//! `qwen-kernels` for the B200 decode engine.
//!
//! The public surface of the reference crate's decoder (`kernels/src/model.rs`: `Model`,
//! `ModelTiles`; `kernels/src/lib.rs:41-49`: `Tile`; `kernels/src/shaders.rs:34`: `MAX_CONTEXT`)
//! over the C ABI of libqne.so (include/qne.h), so that `qwen-agent` builds against this crate
//! unchanged. Methods keep the reference's names, argument meanings, `async` markers and error
//! messages; the work runs on one CUDA device instead of a wgpu adapter. Errors are one type,
//! [`Error`], which implements `std::error::Error + Send + Sync`, so `?` turns it into the
//! `anyhow::Error` the agent uses.

mod ffi;
pub mod model;

use std::ffi::CStr;
use std::fmt;

pub use model::{DeviceSampler, GemvTiming, LoadOptions, Model, ModelTiles};

/// Shader-side constants the agent reads (`kernels/src/shaders.rs:34`).
pub mod shaders {
    /// Upper bound of the attention context in tokens.
    pub const MAX_CONTEXT: u32 = 4096;
}

/// The reference's vocabulary size (`kernels/src/lib.rs`, `VOCAB`).
pub const VOCAB: u32 = 248_320;

/// A GEMV kernel choice of the reference's WGSL kernels (`kernels/src/lib.rs:41-49`). The CUDA
/// kernels choose their own shapes; profiles are validated with the reference's rules and
/// otherwise ignored.
#[derive(Clone, Copy, Debug, PartialEq)]
#[cfg_attr(feature = "serde", derive(serde::Serialize, serde::Deserialize))]
pub struct Tile {
    pub f16: bool,
    pub tpr: u32,
    pub rpw: u32,
    /// Rows per thread group (f16 kernel only).
    pub rpt: u32,
    /// Split-K factor (f16 kernel only).
    pub splits: u32,
}

/// Which class of failure a call hit (the library's `QNE_E*` status codes).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum ErrorKind {
    /// Bad argument or size (`QNE_EINVAL`).
    Invalid,
    /// Context limit of 4096 tokens (`QNE_ERANGE_CTX`).
    ContextLimit,
    /// index.json / weights rejected (`QNE_EFORMAT`).
    Format,
    /// A CUDA call failed (`QNE_ECUDA`).
    Cuda,
    /// A device wait ran past its deadline (`QNE_ETIMEOUT`).
    Timeout,
    /// `restore` without a snapshot (`QNE_ENOSNAP`).
    NoSnapshot,
    /// Device allocation failed (`QNE_ENOMEM`).
    OutOfMemory,
    /// Any other status.
    Other(i32),
}

/// The error of every fallible call: the status and the library's message (the reference's
/// wording, e.g. "context limit of 4096 tokens reached", "no snapshot taken").
#[derive(Clone, Debug)]
pub struct Error {
    pub kind: ErrorKind,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        f.write_str(&self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T, E = Error> = std::result::Result<T, E>;

pub(crate) fn check(status: ffi::qne_status) -> Result<()> {
    if status == ffi::QNE_OK {
        return Ok(());
    }
    let kind = match status {
        ffi::QNE_EINVAL => ErrorKind::Invalid,
        ffi::QNE_ERANGE_CTX => ErrorKind::ContextLimit,
        ffi::QNE_EFORMAT => ErrorKind::Format,
        ffi::QNE_ECUDA => ErrorKind::Cuda,
        ffi::QNE_ETIMEOUT => ErrorKind::Timeout,
        ffi::QNE_ENOSNAP => ErrorKind::NoSnapshot,
        ffi::QNE_ENOMEM => ErrorKind::OutOfMemory,
        other => ErrorKind::Other(other),
    };
    // SAFETY: qne_last_error returns a NUL-terminated thread-local string that stays valid until
    // the next failing call on this thread; it is copied at once.
    let message = unsafe { CStr::from_ptr(ffi::qne_last_error()) }.to_string_lossy().into_owned();
    Err(Error { kind, message })
}

/// Version string of the linked libqne.so.
pub fn engine_version() -> String {
    // SAFETY: a static NUL-terminated string.
    unsafe { CStr::from_ptr(ffi::qne_version()) }.to_string_lossy().into_owned()
}
