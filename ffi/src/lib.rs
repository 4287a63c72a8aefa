//! Rust binding of libmoe_b200, the B200 MoE-layer library (C ABI: include/moe_b200.h).
//!
//! This crate takes the place of moe-680m's Vulkan plumbing (src/device.rs, src/pipeline.rs) for
//! the MoE layer.  `sys` is the raw `extern "C"` block, one declaration per function of the
//! header; `MoeEngine` keeps the reference's own interface for the path:
//!   - `do_route(layer, x_off, m) -> Vec<RoutingOutput>`   (src/inference.rs:622, src/router.rs:4-8)
//!   - `record_and_submit_moe(layer, routing, m, ping) -> Result<(), String>`
//!                                                         (src/inference.rs:663)
//! with the activations in two ping/pong arena buffers, as in the reference's layer loop.
//!
//! NOT COMPILED HERE (the build image has no cargo/rustc).  tests/test_ffi_crate.py checks every
//! declaration below against the C header.

#![allow(non_camel_case_types)]

use std::ffi::c_void;
use std::os::raw::c_char;

pub const MOE_B200_ABI_VERSION: i32 = 1;

pub const MOE_OK: i32 = 0;
pub const MOE_E_INVALID: i32 = -1;
pub const MOE_E_CUDA: i32 = -2;
pub const MOE_E_OOM: i32 = -3;
pub const MOE_E_UNSUPPORTED: i32 = -4;
pub const MOE_E_DEVICE: i32 = -5;

pub const MOE_F_SHARED: u32 = 1;
pub const MOE_F_SHARED_GATE: u32 = 2;
pub const MOE_F_EXPERT_SUBSET: u32 = 4;
pub const MOE_F_REF36: u32 = 8;
pub const MOE_NO_EXPERT: u32 = 0xFFFF_FFFF;

pub const MOE_FT_NO_SHARED: u32 = 1;
pub const MOE_FT_SHARED_ONLY: u32 = 2;
pub const MOE_FT_UNSCALED: u32 = 4;

pub const MOE_EP_TRANSPORT_NCCL: i32 = 0;
pub const MOE_EP_TRANSPORT_PEER: i32 = 1;

pub const MOE_PATH_AUTO: i32 = 0;
pub const MOE_PATH_GEMV: i32 = 1;
pub const MOE_PATH_TC_SMEM_A: i32 = 2;
pub const MOE_PATH_TC_TMEM_A: i32 = 3;

/// Opaque context (`moe_ctx`).
#[repr(C)]
pub struct MoeCtx {
    _private: [u8; 0],
}

/// `moe_layer_spec`: the scalar half of LayerWeights (src/memory.rs:201-223); offsets are arena
/// byte offsets, 0 = missing.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct MoeLayerSpec {
    pub hidden: u32,
    pub inter: u32,
    pub n_experts: u32,
    pub top_k: u32,
    pub flags: u32,
    pub scale: f32,
    pub router_w: u64,
    pub router_bias: u64,
    pub shared_gate: u64,
    pub shared_w1: u64,
    pub shared_w3: u64,
    pub shared_w2: u64,
}

/// `moe_stage_stat`.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct MoeStageStat {
    pub name: [c_char; 24],
    pub calls: u32,
    pub total_ms: f32,
}

pub mod sys {
    use super::*;

    #[link(name = "moe_b200")]
    extern "C" {
        pub fn moe_ctx_create(device: i32, arena_bytes: u64, out: *mut *mut MoeCtx) -> i32;
        pub fn moe_ctx_create_external(device: i32, base: *mut c_void, bytes: u64, out: *mut *mut MoeCtx) -> i32;
        pub fn moe_ctx_destroy(ctx: *mut MoeCtx);
        pub fn moe_arena_upload(ctx: *mut MoeCtx, off: u64, host: *const c_void, n: u64) -> i32;
        pub fn moe_arena_download(ctx: *mut MoeCtx, off: u64, host: *mut c_void, n: u64) -> i32;
        pub fn moe_arena_ptr(ctx: *mut MoeCtx, off: u64, dptr: *mut *mut c_void) -> i32;
        pub fn moe_set_stream(ctx: *mut MoeCtx, stream: *mut c_void) -> i32;
        pub fn moe_sync(ctx: *mut MoeCtx) -> i32;
        pub fn moe_last_error(ctx: *const MoeCtx, buf: *mut c_char, n: usize) -> i32;
        pub fn moe_abi_version() -> i32;
        pub fn moe_layer_create(ctx: *mut MoeCtx, spec: *const MoeLayerSpec, w1: *const u64, w3: *const u64,
                                w2: *const u64, layer_id: *mut u32) -> i32;
        pub fn moe_reserve(ctx: *mut MoeCtx, layer_id: u32, max_tokens: u32) -> i32;
        pub fn moe_route(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, m: u32, topk_off: u64) -> i32;
        pub fn moe_do_route(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, m: u32, routed: *mut u16,
                            weights: *mut f32, shared_gate: *mut f32) -> i32;
        pub fn moe_bucket(ctx: *mut MoeCtx, n_experts: u32, top_k: u32, has_shared: i32, topk_off: u64, m: u32,
                          ranges_off: u64, tokens_off: u64, weights_off: u64, slot_pos_off: u64) -> i32;
        pub fn moe_bucket_static(n_experts: u32, top_k: u32, has_shared: i32, topk: *const c_void, m: u32,
                                 ranges: *mut i32, tokens: *mut i32, weights: *mut f32, slot_pos: *mut i32,
                                 stream: *mut c_void) -> i32;
        pub fn moe_forward(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, resid_off: u64, out_off: u64, m: u32) -> i32;
        pub fn moe_forward_host(ctx: *mut MoeCtx, layer_id: u32, x_host: *const f32, out_host: *mut f32, m: u32,
                                add_residual: i32) -> i32;
        pub fn moe_layer_set_next(ctx: *mut MoeCtx, layer_id: u32, next_id: i32) -> i32;
        pub fn moe_forward_norm(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, out_off: u64, m: u32, eps: f32) -> i32;
        pub fn moe_forward_routed(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, resid_off: u64, out_off: u64,
                                  m: u32, routed: *const u16, weights: *const f32, shared_gate: *const f32) -> i32;
        pub fn moe_forward_topk(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, resid_off: u64, out_off: u64, m: u32,
                                topk_off: u64, flags: u32) -> i32;
        pub fn moe_ep_plan_bytes(m: u32, n_ranks: u32) -> u64;
        pub fn moe_ep_dispatch(ctx: *mut MoeCtx, n_experts: u32, top_k: u32, n_ranks: u32, my_rank: u32,
                               capacity: u32, topk_off: u64, x_off: u64, m: u32, h: u32, plan_off: u64,
                               send_x_off: u64, send_topk_off: u64) -> i32;
        pub fn moe_ep_combine(ctx: *mut MoeCtx, n_ranks: u32, capacity: u32, h: u32, m: u32, plan_off: u64,
                              y_back_off: u64, resid_off: u64, out_off: u64, scale: f32) -> i32;
        pub fn moe_ep_unique_id(out: *mut c_void, n: usize) -> i32;
        pub fn moe_ep_init(ctx: *mut MoeCtx, unique_id: *const c_void, n_ranks: u32, rank: u32) -> i32;
        pub fn moe_forward_ep(ctx: *mut MoeCtx, layer_id: u32, x_off: u64, resid_off: u64, out_off: u64, m: u32,
                              capacity: u32) -> i32;
        pub fn moe_ep_abort(ctx: *mut MoeCtx) -> i32;
        pub fn moe_ep_set_transport(ctx: *mut MoeCtx, transport: i32) -> i32;
        pub fn moe_ep_transport(ctx: *mut MoeCtx, transport: *mut i32) -> i32;
        pub fn moe_set_path(ctx: *mut MoeCtx, path: i32) -> i32;
        pub fn moe_rms_norm(ctx: *mut MoeCtx, x_off: u64, y_off: u64, m: u32, h: u32, eps: f32) -> i32;
        pub fn moe_profile(ctx: *mut MoeCtx, enable: i32) -> i32;
        pub fn moe_profile_read(ctx: *mut MoeCtx, out: *mut MoeStageStat, max: i32, n: *mut i32) -> i32;
        pub fn moe_launch_count(ctx: *mut MoeCtx, n: *mut u64) -> i32;
        pub fn moe_vocab_logits(ctx: *mut MoeCtx, w_off: u64, v: u32, h: u32, x_off: u64, m: u32,
                                logits_off: u64, ids_off: u64) -> i32;
        pub fn moe_silu_mul(ctx: *mut MoeCtx, g_off: u64, u_off: u64, y_off: u64, n: u64) -> i32;
        pub fn moe_dequant_iq4xs(ctx: *mut MoeCtx, src_off: u64, n_blocks: u64, dst_off: u64) -> i32;
        pub fn moe_dequant_ref36(ctx: *mut MoeCtx, src_off: u64, n_blocks: u64, dst_off: u64) -> i32;
        pub fn moe_synth_iq4xs(ctx: *mut MoeCtx, dst_off: u64, key: u64, block_start: u64, n_blocks: u64) -> i32;
    }
}

/// src/router.rs:4-8, unchanged.
#[derive(Clone, Copy, Debug, Default)]
pub struct RoutingOutput {
    pub routed: [u16; 8],
    pub weights: [f32; 8],
    pub shared_id: u16,
}

/// The MoE half of InferenceEngine over the library: one context (arena) and the layer ids in
/// model order.  Not thread-safe, like the reference engine behind its Mutex
/// (src/server.rs:95).
pub struct MoeEngine {
    ctx: *mut MoeCtx,
    pub layer_ids: Vec<u32>,
    pub n_experts: u32,
    pub top_k: u32,
    /// ping/pong hidden-state buffers (arena offsets, f32 [max_tokens][hidden])
    pub hidden_ping: u64,
    pub hidden_pong: u64,
}

fn status(ctx: *const MoeCtx, rc: i32) -> Result<(), String> {
    if rc == MOE_OK {
        return Ok(());
    }
    let mut buf = [0 as c_char; 512];
    unsafe { sys::moe_last_error(ctx, buf.as_mut_ptr(), buf.len()) };
    let msg: Vec<u8> = buf.iter().take_while(|&&c| c != 0).map(|&c| c as u8).collect();
    Err(format!("moe_b200 error {}: {}", rc, String::from_utf8_lossy(&msg)))
}

impl MoeEngine {
    /// DeviceContext::init + allocate_uma (src/device.rs:20, :217): one arena on `device`.
    pub fn new(device: i32, arena_bytes: u64) -> Result<Self, String> {
        let mut ctx: *mut MoeCtx = std::ptr::null_mut();
        status(std::ptr::null(), unsafe { sys::moe_ctx_create(device, arena_bytes, &mut ctx) })?;
        Ok(MoeEngine { ctx, layer_ids: Vec::new(), n_experts: 0, top_k: 0, hidden_ping: 0, hidden_pong: 0 })
    }

    /// load_weights_from_tensors (src/memory.rs:297-321): bytes into the arena at `off`.
    pub fn upload(&self, off: u64, bytes: &[u8]) -> Result<(), String> {
        status(self.ctx, unsafe {
            sys::moe_arena_upload(self.ctx, off, bytes.as_ptr() as *const c_void, bytes.len() as u64)
        })
    }

    /// LayerWeights::from_registry (src/memory.rs:227-290) for one layer: the expert tables are
    /// that layer's slices of expert_w1/w3/w2.
    pub fn add_layer(&mut self, spec: &MoeLayerSpec, w1: &[u64], w3: &[u64], w2: &[u64]) -> Result<u32, String> {
        let n = spec.n_experts as usize;
        if w1.len() != n || w3.len() != n || w2.len() != n {
            return Err(format!("expert tables must hold {} offsets", n));
        }
        let mut id = 0u32;
        status(self.ctx, unsafe {
            sys::moe_layer_create(self.ctx, spec, w1.as_ptr(), w3.as_ptr(), w2.as_ptr(), &mut id)
        })?;
        self.layer_ids.push(id);
        self.n_experts = spec.n_experts;
        self.top_k = spec.top_k;
        Ok(id)
    }

    fn hidden(&self, ping: bool) -> (u64, u64) {
        if ping { (self.hidden_ping, self.hidden_pong) } else { (self.hidden_pong, self.hidden_ping) }
    }

    /// do_route (src/inference.rs:622-659): routing of the m tokens in the current input buffer.
    pub fn do_route(&self, layer: u32, ping: bool, m: u32) -> Result<Vec<RoutingOutput>, String> {
        let k = self.top_k as usize;
        let mut ids = vec![0u16; m as usize * k];
        let mut w = vec![0f32; m as usize * k];
        let (hi, _) = self.hidden(ping);
        status(self.ctx, unsafe {
            sys::moe_do_route(self.ctx, self.layer_ids[layer as usize], hi, m, ids.as_mut_ptr(), w.as_mut_ptr(),
                              std::ptr::null_mut())
        })?;
        Ok((0..m as usize)
            .map(|t| {
                let mut r = RoutingOutput { shared_id: self.n_experts as u16, ..Default::default() };
                r.routed[..k].copy_from_slice(&ids[t * k..t * k + k]);
                r.weights[..k].copy_from_slice(&w[t * k..t * k + k]);
                r
            })
            .collect())
    }

    /// record_and_submit_moe (src/inference.rs:663-766): the MoE layer on the current input with
    /// the given routing, residual included, then the fence wait.  An empty `routing` routes on
    /// the device (moe_forward: router, top-k, bucketing, experts and combine in one call).
    pub fn record_and_submit_moe(&self, layer: u32, routing: &[RoutingOutput], m: u32, ping: bool)
        -> Result<(), String> {
        let id = self.layer_ids[layer as usize];
        let (hi, ho) = self.hidden(ping);
        let rc = if routing.is_empty() {
            unsafe { sys::moe_forward(self.ctx, id, hi, hi, ho, m) }
        } else {
            if routing.len() != m as usize {
                return Err(format!("{} routing rows for {} tokens", routing.len(), m));
            }
            let k = self.top_k as usize;
            let mut ids = Vec::with_capacity(routing.len() * k);
            let mut w = Vec::with_capacity(routing.len() * k);
            for r in routing {
                ids.extend_from_slice(&r.routed[..k]);
                w.extend_from_slice(&r.weights[..k]);
            }
            unsafe {
                sys::moe_forward_routed(self.ctx, id, hi, hi, ho, m, ids.as_ptr(), w.as_ptr(), std::ptr::null())
            }
        };
        status(self.ctx, rc)?;
        status(self.ctx, unsafe { sys::moe_sync(self.ctx) })
    }

    pub fn raw(&self) -> *mut MoeCtx {
        self.ctx
    }
}

impl Drop for MoeEngine {
    fn drop(&mut self) {
        if !self.ctx.is_null() {
            unsafe { sys::moe_ctx_destroy(self.ctx) };
        }
    }
}
