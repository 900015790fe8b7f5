//! Safe wrapper over libgpt2q that keeps the shape of model-lab's CUDA executor
//! (experiments/model-lab/src/gpu.rs): `Gpu::new(&Engine)` (gpu.rs:75), `Gpu::step(tok, pos)`
//! (gpu.rs:212), `Gpu::clear_kv()` (gpu.rs:203) and the `launches` counter (gpu.rs:70).
//!
//! model-lab's `Engine` reaches the wrapper through the `WeightPack` trait, which it implements
//! in a few lines over `Engine::meta`, its tensor records and `Engine::payload` (gpt2.rs:112-119):
//! the library copies every tensor during `new`, so the borrow ends when `new` returns, as in
//! the reference. The panicking methods mirror the reference's `expect` behaviour; every one has
//! a `try_` twin that returns the library's status and message instead.
use std::ffi::{CStr, CString};
use std::fmt;
use std::os::raw::c_int;
use std::ptr;

use gpt2q_sys as sys;

/// A failed library call: the status code (GPT2Q_E*) and `gpt2q_last_error`.
#[derive(Debug, Clone)]
pub struct Error {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "gpt2q error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

/// Architecture of a pack (gpt2.rs:11-19 `Meta`).
#[derive(Debug, Clone, Copy)]
pub struct Meta {
    pub n_embd: usize,
    pub n_layer: usize,
    pub n_head: usize,
    pub n_ctx: usize,
    pub vocab: usize,
    pub ln_eps: f32,
}

/// One tensor as stored in the pack's TENSORS section: name, atom, shape ([out, in] for 2-D
/// weights) and the payload bytes.
pub struct TensorView<'a> {
    pub name: &'a str,
    pub atom: &'a str,
    pub shape: &'a [usize],
    pub payload: &'a [u8],
}

/// What `Gpu::new` needs from a weight container; model-lab's `Engine` implements it.
pub trait WeightPack {
    fn meta(&self) -> Meta;
    fn tensors(&self) -> Vec<TensorView<'_>>;
}

fn last_error(h: *const sys::gpt2q_handle) -> String {
    unsafe {
        let p = sys::gpt2q_last_error(h);
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

fn check(h: *const sys::gpt2q_handle, rc: c_int) -> Result<()> {
    if rc == sys::GPT2Q_OK {
        Ok(())
    } else {
        Err(Error { code: rc, message: last_error(h) })
    }
}

/// One GPU's handle: weights in HBM, a KV cache for `max_seqs` sequences.
pub struct Gpu {
    h: *mut sys::gpt2q_handle,
    vocab: usize,
    n_ctx: usize,
    /// Kernel launches so far (gpu.rs:70), refreshed after every call.
    pub launches: u64,
}

// A handle may move between threads; it must not be used from two at once (it is not Sync).
unsafe impl Send for Gpu {}

impl Gpu {
    /// Gpu::new(&Engine) (gpu.rs:75): device 0, one sequence, panics on failure.
    pub fn new<P: WeightPack>(pack: &P) -> Self {
        Self::try_new(pack, 0, 1, 0).unwrap_or_else(|e| panic!("gpt2q_create: {e}"))
    }

    /// Uploads every tensor of `pack` to `device`, with KV slots for `max_seqs` sequences and a
    /// prefill workspace of `max_tokens` tokens (0 = the library's default).
    pub fn try_new<P: WeightPack>(pack: &P, device: i32, max_seqs: i32, max_tokens: i32) -> Result<Self> {
        let m = pack.meta();
        let cfg = sys::gpt2q_config {
            n_embd: m.n_embd as i32,
            n_layer: m.n_layer as i32,
            n_head: m.n_head as i32,
            n_ctx: m.n_ctx as i32,
            vocab: m.vocab as i32,
            ln_eps: m.ln_eps,
            max_seqs,
            max_tokens,
        };
        let views = pack.tensors();
        let names: Vec<(CString, CString)> = views
            .iter()
            .map(|t| (CString::new(t.name).expect("tensor name"), CString::new(t.atom).expect("atom name")))
            .collect();
        let mut descs = Vec::with_capacity(views.len());
        for (t, (n, a)) in views.iter().zip(&names) {
            if t.shape.is_empty() || t.shape.len() > 2 {
                return Err(Error { code: sys::GPT2Q_EARG, message: format!("tensor {}: rank must be 1 or 2", t.name) });
            }
            let mut shape = [0i64; 2];
            for (i, s) in t.shape.iter().enumerate() {
                shape[i] = *s as i64;
            }
            descs.push(sys::gpt2q_tensor_desc {
                name: n.as_ptr(),
                atom: a.as_ptr(),
                ndim: t.shape.len() as i32,
                shape,
                data: t.payload.as_ptr() as *const _,
                len: t.payload.len() as u64,
            });
        }
        let mut h = ptr::null_mut();
        let rc = unsafe { sys::gpt2q_create(&cfg, descs.as_ptr(), descs.len() as c_int, device, &mut h) };
        check(ptr::null(), rc)?;
        Ok(Gpu { h, vocab: m.vocab, n_ctx: m.n_ctx, launches: 0 })
    }

    fn refresh(&mut self) {
        self.launches = unsafe { sys::gpt2q_launches(self.h) };
    }

    /// Gpu::step (gpu.rs:212): token `tok` of sequence slot 0 at `pos`; the vocab logits.
    pub fn step(&mut self, tok: u32, pos: usize) -> Vec<f32> {
        self.try_step(tok, pos).unwrap_or_else(|e| panic!("gpt2q_step: {e}"))
    }

    pub fn try_step(&mut self, tok: u32, pos: usize) -> Result<Vec<f32>> {
        let mut out = vec![0f32; self.vocab];
        let rc = unsafe { sys::gpt2q_step(self.h, tok, pos as i32, out.as_mut_ptr()) };
        self.refresh();
        check(self.h, rc).map(|_| out)
    }

    /// Gpu::clear_kv (gpu.rs:203): every slot.
    pub fn clear_kv(&mut self) {
        let rc = unsafe { sys::gpt2q_reset_kv(self.h, ptr::null(), 0) };
        check(self.h, rc).unwrap_or_else(|e| panic!("gpt2q_reset_kv: {e}"));
    }

    /// Engine::step batched over sequences: sequence i feeds tok[i] at pos[i] into slot i;
    /// returns the greedy next token of each.
    pub fn decode(&mut self, tok: &[u32], pos: &[i32]) -> Result<Vec<u32>> {
        assert_eq!(tok.len(), pos.len());
        let mut next = vec![0u32; tok.len()];
        let rc = unsafe {
            sys::gpt2q_decode(self.h, tok.as_ptr(), pos.as_ptr(), ptr::null(), tok.len() as c_int,
                              ptr::null_mut(), next.as_mut_ptr())
        };
        self.refresh();
        check(self.h, rc).map(|_| next)
    }

    /// The prompt loop of generate_greedy (gpt2.rs:373-381) for many prompts in one pass:
    /// prompt i goes to slot i; returns the logits of every prompt's last position
    /// ([n][vocab], row-major) and the greedy next tokens.
    pub fn prefill(&mut self, prompts: &[&[u32]]) -> Result<(Vec<f32>, Vec<u32>)> {
        let (toks, offs) = flatten(prompts);
        let mut logits = vec![0f32; prompts.len() * self.vocab];
        let mut next = vec![0u32; prompts.len()];
        let rc = unsafe {
            sys::gpt2q_prefill(self.h, toks.as_ptr(), offs.as_ptr(), ptr::null(), prompts.len() as c_int,
                               logits.as_mut_ptr(), next.as_mut_ptr())
        };
        self.refresh();
        check(self.h, rc).map(|_| (logits, next))
    }

    /// generate_greedy (gpt2.rs:367-388) for every prompt: `steps` tokens each ([n][steps];
    /// u32::MAX where a sequence reached n_ctx).
    pub fn generate_greedy(&mut self, prompts: &[&[u32]], steps: usize) -> Result<Vec<u32>> {
        let (toks, offs) = flatten(prompts);
        let mut out = vec![0u32; prompts.len() * steps];
        let rc = unsafe {
            sys::gpt2q_generate_greedy(self.h, toks.as_ptr(), offs.as_ptr(), prompts.len() as c_int,
                                       steps as c_int, out.as_mut_ptr())
        };
        self.refresh();
        check(self.h, rc).map(|_| out)
    }

    /// nll_per_token (gpt2.rs:347-364) on the device; overwrites the KV cache of `slot`.
    pub fn nll(&mut self, ids: &[u32], slot: i32) -> Result<f64> {
        let mut out = 0f64;
        let rc = unsafe { sys::gpt2q_nll(self.h, ids.as_ptr(), ids.len() as c_int, slot, &mut out) };
        self.refresh();
        check(self.h, rc).map(|_| out)
    }

    /// Gpu::set_adapter (gpu.rs:188-194): a [r][d], b [d][r] row-major.
    pub fn set_adapter(&mut self, a: &[f32], b: &[f32], r: usize) -> Result<()> {
        let rc = unsafe { sys::gpt2q_set_adapter(self.h, a.as_ptr(), b.as_ptr(), r as c_int) };
        check(self.h, rc)
    }

    /// Gpu::clear_adapter (gpu.rs:195).
    pub fn clear_adapter(&mut self) -> Result<()> {
        let rc = unsafe { sys::gpt2q_clear_adapter(self.h) };
        check(self.h, rc)
    }

    pub fn n_ctx(&self) -> usize {
        self.n_ctx
    }
}

impl Drop for Gpu {
    fn drop(&mut self) {
        unsafe { sys::gpt2q_destroy(self.h) }
    }
}

fn flatten(prompts: &[&[u32]]) -> (Vec<u32>, Vec<i32>) {
    let mut toks = Vec::new();
    let mut offs = Vec::with_capacity(prompts.len() + 1);
    offs.push(0i32);
    for p in prompts {
        toks.extend_from_slice(p);
        offs.push(toks.len() as i32);
    }
    (toks, offs)
}
