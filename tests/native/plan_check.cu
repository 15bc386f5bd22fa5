// Host-side exhaustive check of the tensor-core ancestor kernel's tile planner
// (qattention_b200/csrc/ancestor_plan.cuh), compiled and run by
// tests/test_tile_plan.py. For many complete trees (branching 2-16, depths up
// to 12, truncated sequences, several max_depth values) and both tilings it
// checks that: every node is a query of exactly one tile; tiles hold at most
// 64 rows; windows are disjoint and in descending node order; every node of
// a warp's key windows is staged by its tile (so each key column maps to a
// shared-memory row); every node of every row's ancestor walk (the
// reference's parent rule, duplicates ending the walk at the root) lies in
// its warp's windows where the kernel's forward scan finds it; and the
// capacities the host computes bound every tile and warp.
#include "../../qattention_b200/csrc/ancestor_plan.cuh"
#include <cstdio>
#include <vector>
#include <set>
using namespace qa;
static int F(int b, int L){ long f=0; for(int i=0;i<L;i++) f=f*b+1; return (int)f; }
int fails=0;
#define CHECK(c, ...) do{ if(!(c)){ if(fails<20) {printf(__VA_ARGS__); printf("\n");} ++fails; } }while(0)
bool in_windows(const int* wl, const int* wb, int nw, int node, int& slot){
  for(int i=0;i<nw;i++){ int hi = wl[i] + (wb[i+1]-wb[i]) - 1; if(node>=wl[i] && node<=hi){ slot = wb[i] + node - wl[i]; return true;} }
  return false;
}
void check(int b, int n, int max_depth, bool sub){
  TileGeom g = make_tile_geom(b, n, sub);
  int rows_cap, keys_cap; tile_geom_caps(g, n, max_depth, rows_cap, keys_cap);
  for (int len : {n, n - 1, n / 2 + 1, 1}) {
    if (len < 1) continue;
    std::vector<int> cover(len, 0);
    for(int t=0;t<g.tiles;t++){
      int seg_lo[kMaxLevels+1], seg_row[kMaxLevels+2];
      int ns = tile_segments(g,t,len,seg_lo,seg_row);
      int rows = seg_row[ns];
      CHECK(rows <= kTileRows, "rows>64 b=%d n=%d t=%d", b,n,t);
      if(rows==0) continue;
      std::vector<int> node(rows);
      for(int r=0;r<rows;r++){ int i=0; while(seg_row[i+1]<=r) ++i; node[r]=seg_lo[i]+r-seg_row[i];
        CHECK(node[r]>=0 && node[r]<len, "node oob"); if(node[r]>=0&&node[r]<len) cover[node[r]]++; }
      int wl[kMaxWin+1], wb[kMaxWin+1], nw;
      int tot = plan_rows(g,seg_lo,seg_row,ns,0,rows,max_depth,HostDivB{(uint32_t)b},wl,wb,nw);
      CHECK(tot <= rows_cap, "cta rows %d > cap %d", tot, rows_cap);
      CHECK(tot == wb[nw], "total mismatch");
      for(int i=0;i+1<nw;i++){ int hi1 = wl[i+1] + (wb[i+2]-wb[i+1]) - 1; CHECK(hi1 < wl[i]-1, "windows not descending/disjoint b=%d n=%d t=%d",b,n,t); }
      for(int i=0;i<nw;i++) { int hi = wl[i] + (wb[i+1]-wb[i]) - 1; CHECK(wl[i]>=0 && hi < len, "window node oob b=%d n=%d len=%d t=%d [%d,%d]", b,n,len,t,wl[i],hi); }
      for(int w=0; w*16<rows; w++){
        int r0=16*w, r1=std::min(rows,16*w+16);
        int xl[kMaxWin+1], xb[kMaxWin+1], xn;
        int keys = plan_rows(g,seg_lo,seg_row,ns,r0,r1,max_depth,HostDivB{(uint32_t)b},xl,xb,xn);
        CHECK(keys <= keys_cap, "keys %d > cap %d", keys, keys_cap);
        for(int i=0;i+1<xn;i++){ int hi1 = xl[i+1] + (xb[i+2]-xb[i+1]) - 1; CHECK(hi1 < xl[i]-1, "warp windows not descending"); }
        // every warp window node inside CTA windows
        for(int i=0;i<xn;i++){ int hi = xl[i] + (xb[i+1]-xb[i]) - 1; for(int v=xl[i]; v<=hi; v++){ int s; CHECK(in_windows(wl,wb,nw,v,s), "warp node %d not staged b=%d n=%d t=%d",v,b,n,t); if(in_windows(wl,wb,nw,v,s)) CHECK(s<tot,"slot"); } }
        // walk keys inside warp windows (and the kernel's monotone scan finds them)
        for(int r=r0;r<r1;r++){
          int v=node[r], wi=0;
          for(int s=0;s<=max_depth;s++){
            if(s>0){ if(v==0) break; v=(v-1)/b; }
            while(wi+1<xn && v<xl[wi]) ++wi;
            int hi = xl[wi] + (xb[wi+1]-xb[wi]) - 1;
            CHECK(v>=xl[wi] && v<=hi, "walk node %d not in warp window b=%d n=%d t=%d r=%d s=%d", v,b,n,t,r,s);
          }
        }
      }
    }
    for(int v=0; v<len; v++) CHECK(cover[v]==1, "node %d covered %d times b=%d n=%d len=%d sub=%d", v, cover[v], b,n,len,sub);
  }
}
int main(){
  int shapes=0;
  for(int b=2;b<=16;b++) for(int d=0; d<=12; d++){
    long N = F(b,d+1); if(N> 70000) break;
    for(int md : {d, 0, 1, 2, d>3?d-2:d, 40}) for(int sub=0;sub<2;sub++){ check(b,(int)N,md,sub); shapes++; }
    if (N > 5) for(int sub=0;sub<2;sub++){ check(b,(int)N-3,d,sub); check(b,(int)N/2+7 > (int)N ? (int)N : (int)N/2+7,d,sub); }
  }
  // the benchmark shapes: report caps
  struct {int b,d;} cs[] = {{2,3},{4,5},{2,9},{4,4},{3,6},{8,3},{2,12}};
  for(auto c: cs){ int N=F(c.b,c.d+1); for(int sub=0;sub<2;sub++){ TileGeom g=make_tile_geom(c.b,N,sub); int rc,kc; tile_geom_caps(g,N,c.d,rc,kc); printf("b=%d d=%d N=%d sub=%d(bands=%d h=%d k=%d) tiles=%d rows_cap=%d keys_cap=%d\n",c.b,c.d,N,sub,g.bands,g.bands?g.band_h[g.bands-1]:0,g.bands?g.band_k[g.bands-1]:0,g.tiles,rc,kc);} }
  printf("shapes %d fails %d\n", shapes, fails);
  return fails!=0;
}
