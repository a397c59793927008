//! Links libfa_attn.so from FA_ATTN_DIR (the directory the library was built into; in this
//! repository `fusor-ai_b200/fusor_attn`).
fn main() {
    println!("cargo:rerun-if-env-changed=FA_ATTN_DIR");
    if let Ok(dir) = std::env::var("FA_ATTN_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
    }
    println!("cargo:rustc-link-lib=dylib=fa_attn");
}
