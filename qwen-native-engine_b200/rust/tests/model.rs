//! The façade against libqne.so: tile profiles and load-time rejections need no GPU; the decode
//! test runs when QNE_TEST_MODEL_DIR names a directory with index.json and weights.bin (for
//! example one written by `qne.synth.build(...).save(dir)`) and a B200 is present.
use std::future::Future;
use std::pin::pin;
use std::task::{Context, Poll, RawWaker, RawWakerVTable, Waker};

use qwen_kernels::{ErrorKind, LoadOptions, Model, ModelTiles, Tile};

/// The façade's futures complete on their first poll (the library call blocks), so a one-poll
/// executor stands in for pollster here.
fn block_on<F: Future>(f: F) -> F::Output {
    fn noop(_: *const ()) {}
    fn clone(p: *const ()) -> RawWaker {
        RawWaker::new(p, &VTABLE)
    }
    static VTABLE: RawWakerVTable = RawWakerVTable::new(clone, noop, noop, noop);
    // SAFETY: the vtable's functions do nothing with the null data pointer.
    let waker = unsafe { Waker::from_raw(RawWaker::new(std::ptr::null(), &VTABLE)) };
    let mut cx = Context::from_waker(&waker);
    let mut f = pin!(f);
    match f.as_mut().poll(&mut cx) {
        Poll::Ready(v) => v,
        Poll::Pending => panic!("a façade future did not complete on its first poll"),
    }
}

#[test]
fn tile_profiles_follow_the_reference_rules() {
    assert!(ModelTiles::fast().validate().is_ok());
    assert!(ModelTiles::f32().validate().is_ok());
    let mut bad = ModelTiles::fast();
    bad.down = Tile { f16: false, tpr: 16, rpw: 4, rpt: 2, splits: 1 };
    let e = bad.validate().unwrap_err();
    assert_eq!(e.kind, ErrorKind::Format);
    assert!(e.message.starts_with("invalid kernel tile profile"), "{}", e.message);
}

#[test]
fn load_rejects_what_the_reference_rejects() {
    let index = r#"{"config":{"layers":4,"full_attention_every":4,"hidden":1024,"intermediate":3584,
        "vocab":512,"rope_theta":10000000.0,"rope_dim":64},"matrices":{},"tensors":{}}"#;
    let e = block_on(Model::load(index, &[0u8; 64], ModelTiles::fast(), true, None)).err().unwrap();
    assert_eq!(e.kind, ErrorKind::Format);
    assert_eq!(e.message, "unsupported model architecture: these kernels require Qwen3.5-0.8B or Qwen3.5-2B");
    let e = block_on(Model::load("{", &[], ModelTiles::fast(), true, None)).err().unwrap();
    assert_eq!(e.kind, ErrorKind::Format);
}

#[test]
fn decode_snapshot_restore_on_a_gpu() {
    let Ok(dir) = std::env::var("QNE_TEST_MODEL_DIR") else { return };
    let index = std::fs::read_to_string(format!("{dir}/index.json")).unwrap();
    let weights = std::fs::read(format!("{dir}/weights.bin")).unwrap();
    let m = Model::load_with(&index, &weights, LoadOptions { device: 0, any_shape: true }).unwrap();
    drop(weights);
    assert!(m.adapter.contains("sm_10"), "{}", m.adapter);
    let prompt: Vec<u32> = (0..24u32).map(|i| (i * 7919 + 13) % 512).collect();
    block_on(m.prefill_chunk(&prompt, 0, true)).unwrap();
    let logits = block_on(m.logits()).unwrap();
    let (tok, pos) = block_on(m.last_token()).unwrap();
    assert_eq!(pos, prompt.len() as u32);
    let best = (0..logits.len()).max_by(|&a, &b| logits[a].total_cmp(&logits[b]).then(b.cmp(&a))).unwrap();
    assert_eq!(tok as usize, best);
    m.snapshot();
    let a = block_on(m.decode(8, 1, &[])).unwrap();
    m.restore().unwrap();
    let b = block_on(m.decode(8, 1, &[])).unwrap();
    assert_eq!(a, b);
    let e = block_on(m.step(1, 4096)).err().unwrap();
    assert_eq!(e.kind, ErrorKind::ContextLimit);
    let prof = block_on(m.profile_token()).unwrap();
    assert!(prof.contains_key("gdn") && prof.contains_key("attention"), "{prof:?}");
    assert_eq!(m.dispatches_per_token(), 5 * 4 + 1);
}
