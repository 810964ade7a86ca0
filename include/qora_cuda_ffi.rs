// FFI binding of include/qora_cuda.h.  Link with -lqora_b200 -lcudart.
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub const QORA_OK: c_int = 0;

#[repr(C)] pub struct qora_ctx { _p: [u8; 0] }
#[repr(C)] pub struct qora_w4 { _p: [u8; 0] }
#[repr(C)] pub struct qora_kv { _p: [u8; 0] }
#[repr(C)] pub struct qora_talker { _p: [u8; 0] }
#[repr(C)] pub struct qora_predictor { _p: [u8; 0] }
#[repr(C)] pub struct qora_engine { _p: [u8; 0] }
#[repr(C)] pub struct qora_text_proj { _p: [u8; 0] }
#[repr(C)] pub struct qora_model_file { _p: [u8; 0] }
#[repr(C)] pub struct qora_decoder { _p: [u8; 0] }

/// qora_decoder_dims: SpeechDecoderWeights' configuration (decoder.rs:56-66).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct qora_decoder_dims {
    pub codebook_dim: i32, pub codebook_size: i32, pub num_quantizers: i32, pub vq_dim: i32,
    pub latent: i32, pub hidden: i32, pub num_heads: i32, pub head_dim: i32,
    pub intermediate: i32, pub num_layers: i32, pub sliding_window: i32,
    pub upsample_stages: i32, pub upsample_inner: i32, pub vocos_blocks: i32,
    pub vocos_channels: [i32; 8], pub vocos_kernels: [i32; 8], pub vocos_strides: [i32; 8],
    pub rope_max_pos: i32, pub rope_theta: f64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct qora_q4_host {
    pub packed: *const u8,   // Q4Weight::packed
    pub scales: *const u16,  // Q4Weight::scales (f16 bits)
    pub k: i64,
    pub n: i64,
}

#[repr(C)]
pub struct qora_layer_host {
    pub q_proj: qora_q4_host, pub k_proj: qora_q4_host, pub v_proj: qora_q4_host,
    pub o_proj: qora_q4_host, pub gate_proj: qora_q4_host, pub up_proj: qora_q4_host,
    pub down_proj: qora_q4_host,
    pub q_norm: *const u16, pub k_norm: *const u16,
    pub input_norm: *const u16, pub post_attn_norm: *const u16,
}

#[repr(C)]
pub struct qora_talker_host {
    pub num_layers: i32, pub hidden: i32, pub num_heads: i32, pub num_kv_heads: i32,
    pub head_dim: i32, pub ffn: i32, pub vocab: i32, pub rope_max_pos: i32,
    pub rope_theta: f64,
    pub layers: *const qora_layer_host,
    pub codec_embedding: qora_q4_host,
    pub codec_head: qora_q4_host,
    pub final_norm: *const u16,
}

#[repr(C)]
pub struct qora_predictor_host {
    pub num_layers: i32, pub hidden: i32, pub num_heads: i32, pub num_kv_heads: i32,
    pub head_dim: i32, pub ffn: i32, pub vocab: i32, pub num_groups: i32,
    pub rope_max_pos: i32, pub rope_theta: f64,
    pub layers: *const qora_layer_host,
    pub input_proj: qora_q4_host,          // packed == null => identity
    pub input_proj_bias: *const f32,
    pub codec_embeddings: *const qora_q4_host,
    pub lm_heads: *const qora_q4_host,
    pub final_norm: *const u16,
}

#[repr(C)]
pub struct qora_text_proj_host {
    pub text_embedding: qora_q4_host,      // [text_vocab][text_hidden]
    pub fc1: qora_q4_host,                 // text_projection.linear_fc1
    pub fc2: qora_q4_host,                 // text_projection.linear_fc2
    pub fc1_bias: *const f32,
    pub fc2_bias: *const f32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct qora_prompt_row {
    pub text: i32,          // row of text_rows, or -1
    pub codes_n: i32,       // 0 none, 1 codec token, 16 reference frame, -1 voice
    pub codes: [u32; 16],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct qora_sample_params {
    pub temperature: f32, pub top_k: i32, pub top_p: f32, pub repetition_penalty: f32,
}

#[link(name = "qora_b200")]
extern "C" {
    pub fn qora_ctx_create(device: i32, out: *mut *mut qora_ctx) -> c_int;
    pub fn qora_ctx_destroy(ctx: *mut qora_ctx);
    pub fn qora_status_string(status: i32) -> *const c_char;
    pub fn qora_last_error() -> *const c_char;
    pub fn qora_ctx_check_device_error(ctx: *mut qora_ctx, stream: *mut c_void) -> c_int;

    pub fn qora_q4_quantize_host(data: *const f32, k: i64, n: i64, packed: *mut u8,
                                 scales: *mut u16) -> c_int;
    pub fn qora_synth_normal_host(seed: u64, sigma: f32, count: i64, out: *mut f32) -> c_int;
    pub fn qora_synth_q4_host(seed: u64, sigma: f32, k: i64, n: i64, packed: *mut u8,
                              scales: *mut u16) -> c_int;
    pub fn qora_q4_weight_upload(ctx: *mut qora_ctx, w: *const qora_q4_host,
                                 out: *mut *mut qora_w4) -> c_int;
    pub fn qora_q4_weight_destroy(w: *mut qora_w4);
    pub fn qora_q4_gemv(ctx: *mut qora_ctx, w: *const qora_w4, x: *const f32, y: *mut f32,
                        batch: i32, stream: *mut c_void) -> c_int;
    pub fn qora_q4_gemm(ctx: *mut qora_ctx, w: *const qora_w4, x: *const f32, seq_len: i64,
                        y: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_q4_embed_rows(ctx: *mut qora_ctx, w: *const qora_w4, tokens: *const u32,
                              count: i32, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_rms_norm_f16(ctx: *mut qora_ctx, x: *const f32, gamma: *const u16, n: i64,
                             rows: i32, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_rope_tables_host(head_dim: i32, max_pos: i32, theta: f64, sections: *const i32,
                                 n_sections: i32, cos: *mut f32, sin: *mut f32) -> c_int;

    pub fn qora_kv_create(ctx: *mut qora_ctx, num_layers: i32, kv_heads: i32, head_dim: i32,
                          max_pos: i32, streams: i32, out: *mut *mut qora_kv) -> c_int;
    pub fn qora_kv_create_paged(ctx: *mut qora_ctx, num_layers: i32, kv_heads: i32, head_dim: i32,
                                max_pos: i32, streams: i32, page_positions: i32, pool_pages: i32,
                                out: *mut *mut qora_kv) -> c_int;
    pub fn qora_kv_pages_host(kv: *const qora_kv, mapped: *mut i32, free_pages: *mut i32) -> c_int;
    pub fn qora_kv_destroy(kv: *mut qora_kv);
    pub fn qora_kv_reset(kv: *mut qora_kv, ids: *const i32, count: i32,
                         stream: *mut c_void) -> c_int;
    pub fn qora_kv_lengths_host(kv: *mut qora_kv, len: *mut i32, stream: *mut c_void) -> c_int;
    pub fn qora_kv_copy_stream(dst: *mut qora_kv, dst_stream: i32, src: *const qora_kv,
                               src_stream: i32, stream: *mut c_void) -> c_int;
    pub fn qora_kv_layer_ptrs(kv: *mut qora_kv, layer: i32, k: *mut *mut f32,
                              v: *mut *mut f32, len: *mut *mut i32) -> c_int;
    pub fn qora_kv_export_layer(kv: *mut qora_kv, layer: i32, k_out: *mut f32,
                                v_out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_kv_attend(kv: *mut qora_kv, layer: i32, qkv: *const f32, num_heads: i32,
                          q_norm: *const u16, k_norm: *const u16, rope_cos: *const f32,
                          rope_sin: *const f32, rope_max_pos: i32, positions: *const i32,
                          b: i32, advance: i32, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_kv_attend_noalloc(kv: *mut qora_kv, layer: i32, qkv: *const f32,
                                  num_heads: i32, q_norm: *const u16, k_norm: *const u16,
                                  rope_cos: *const f32, rope_sin: *const f32,
                                  rope_max_pos: i32, positions: *const i32, b: i32,
                                  advance: i32, out: *mut f32, stream: *mut c_void) -> c_int;

    pub fn qora_talker_create(ctx: *mut qora_ctx, host: *const qora_talker_host,
                              max_batch: i32, out: *mut *mut qora_talker) -> c_int;
    pub fn qora_talker_destroy(t: *mut qora_talker);
    pub fn qora_talker_step(t: *mut qora_talker, kv: *mut qora_kv, emb: *const f32,
                            positions: *const i32, b: i32, hidden: *mut f32, logits: *mut f32,
                            stream: *mut c_void) -> c_int;
    pub fn qora_talker_prefill(t: *mut qora_talker, kv: *mut qora_kv, kv_stream: i32,
                               x: *const f32, t_len: i32, start_pos: i32, hidden: *mut f32,
                               stream: *mut c_void) -> c_int;
    pub fn qora_talker_decode(t: *mut qora_talker, kv: *mut qora_kv, tp: *mut qora_text_proj,
                              tokens_host: *const u32, is_text: i32, positions: *const i32,
                              b: i32, hidden: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_talker_codec_head(t: *mut qora_talker, hidden: *const f32, b: i32,
                                  logits: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qora_talker_embed_codec(t: *mut qora_talker, tokens: *const u32, b: i32,
                                   out: *mut f32, stream: *mut c_void) -> c_int;

    pub fn qora_model_file_open(path: *const c_char, out: *mut *mut qora_model_file) -> c_int;
    pub fn qora_model_file_talker(f: *const qora_model_file, out: *mut qora_talker_host) -> c_int;
    pub fn qora_model_file_predictor(f: *const qora_model_file,
                                     out: *mut qora_predictor_host) -> c_int;
    pub fn qora_model_file_text_proj(f: *const qora_model_file,
                                     out: *mut qora_text_proj_host) -> c_int;
    pub fn qora_model_file_close(f: *mut qora_model_file);

    pub fn qora_text_proj_create(ctx: *mut qora_ctx, host: *const qora_text_proj_host,
                                 out: *mut *mut qora_text_proj) -> c_int;
    pub fn qora_text_proj_destroy(tp: *mut qora_text_proj);
    pub fn qora_text_proj_embed(tp: *mut qora_text_proj, tokens_host: *const u32, count: i32,
                                out: *mut f32, stream: *mut c_void) -> c_int;

    pub fn qora_prompt_assemble(t: *mut qora_talker, p: *mut qora_predictor,
                                text_rows: *const f32, n_text: i32, voice: *const f32,
                                voice_len: i32, rows: *const qora_prompt_row, count: i32,
                                out: *mut f32, stream: *mut c_void) -> c_int;

    pub fn qora_predictor_create(ctx: *mut qora_ctx, host: *const qora_predictor_host,
                                 max_batch: i32, out: *mut *mut qora_predictor) -> c_int;
    pub fn qora_predictor_destroy(p: *mut qora_predictor);
    pub fn qora_predictor_frame(p: *mut qora_predictor, kv: *mut qora_kv, hidden: *const f32,
                                semantic: *const f32, b: i32, codes: *mut u32,
                                logits: *mut f32, forced: *const u32,
                                stream: *mut c_void) -> c_int;
    pub fn qora_predictor_embed_sum(p: *mut qora_predictor, codes: *const u32, b: i32,
                                    out: *mut f32, stream: *mut c_void) -> c_int;

    pub fn qora_sample(ctx: *mut qora_ctx, logits: *const f32, b: i32, v: i32,
                       prev: *const u32, n_prev: i32, rng: *mut u64,
                       params: *const qora_sample_params, out: *mut u32,
                       stream: *mut c_void) -> c_int;

    pub fn qora_engine_create(t: *mut qora_talker, p: *mut qora_predictor, b: i32,
                              max_pos: i32, params: *const qora_sample_params,
                              out: *mut *mut qora_engine) -> c_int;
    pub fn qora_engine_destroy(e: *mut qora_engine);
    pub fn qora_engine_prefill(e: *mut qora_engine, x_host: *const f32, t_len: i32,
                               seeds_host: *const u64, stream: *mut c_void) -> c_int;
    pub fn qora_engine_prefill_from(e: *mut qora_engine, prefix: *const qora_kv,
                                    prefix_stream: i32, prefix_len: i32, x_host: *const f32,
                                    t_len: i32, seeds_host: *const u64,
                                    stream: *mut c_void) -> c_int;
    pub fn qora_engine_frame(e: *mut qora_engine, text: *const f32, codes: *mut u32,
                             stream: *mut c_void) -> c_int;
    pub fn qora_engine_frame_host(e: *mut qora_engine, text_host: *const f32,
                                  codes_host: *mut u32, stream: *mut c_void) -> c_int;
    pub fn qora_engine_use_graph(e: *mut qora_engine, enable: i32) -> c_int;
    pub fn qora_engine_use_persistent(e: *mut qora_engine, enable: i32) -> c_int;
    pub fn qora_engine_set_temperature(e: *mut qora_engine, temperature: f32) -> c_int;
    pub fn qora_engine_trace(e: *mut qora_engine, enable: i32, capacity: i32, n_ops: *mut i32,
                             ops_host: *mut i32, stamps_host: *mut u64) -> c_int;
    pub fn qora_engine_kernels_per_frame(e: *mut qora_engine, count: *mut i32) -> c_int;
    pub fn qora_engine_state(e: *mut qora_engine, logits: *mut *mut f32, hidden: *mut *mut f32,
                             prev: *mut *mut u32, rng: *mut *mut u64,
                             positions: *mut *mut i32) -> c_int;

    // load_speech_decoder (loader.rs:503-716): one set_tensor per safetensors tensor
    pub fn qora_decoder_create(ctx: *mut qora_ctx, dims: *const qora_decoder_dims,
                               out: *mut *mut qora_decoder) -> c_int;
    pub fn qora_decoder_set_tensor(dec: *mut qora_decoder, name: *const c_char,
                                   data_host: *const f32, count: i64) -> c_int;
    pub fn qora_decoder_finalize(dec: *mut qora_decoder) -> c_int;
    pub fn qora_decoder_destroy(dec: *mut qora_decoder);
    pub fn qora_model_file_decoder(f: *const qora_model_file, ctx: *mut qora_ctx,
                                   out: *mut *mut qora_decoder) -> c_int;
    pub fn qora_decoder_get_dims(dec: *const qora_decoder, dims: *mut qora_decoder_dims) -> c_int;
    pub fn qora_decoder_use_tensor_cores(dec: *mut qora_decoder, mode: i32) -> c_int;
    pub fn qora_decoder_samples(dec: *const qora_decoder, frames: i64, samples: *mut i64) -> c_int;
    // decode_to_audio (decoder.rs:395-582)
    pub fn qora_decode_to_audio(dec: *mut qora_decoder, codes_host: *const u32, frames: i64,
                                warmup_host: *const u32, warmup_frames: i64,
                                samples_host: *mut f32, capacity: i64, n_samples: *mut i64,
                                stream: *mut c_void) -> c_int;
    pub fn qora_decode_to_audio_device(dec: *mut qora_decoder, codes: *const u32, frames: i64,
                                       warmup_frames: i64, samples: *mut f32, launches: *mut i32,
                                       stream: *mut c_void) -> c_int;
}

/// Turns a status into a Result with the library's message (the reference
/// panics where these return an error).
pub fn check(rc: c_int) -> Result<(), String> {
    if rc == QORA_OK { return Ok(()); }
    let msg = unsafe { std::ffi::CStr::from_ptr(qora_last_error()) };
    Err(format!("qora: {} ({})",
        unsafe { std::ffi::CStr::from_ptr(qora_status_string(rc)) }.to_string_lossy(),
        msg.to_string_lossy()))
}
